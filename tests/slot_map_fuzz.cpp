// Randomised comparison of kvp::SlotMap (the streaming manager's row -> slot
// table) with std::unordered_map: puts, erases (backward-shift deletion),
// finds, the LONG_MIN key, periodic clears.  Built and run by
// tests/test_slot_map.py.
#include "slot_map.h"
#include <unordered_map>
#include <random>
#include <cstdio>
#include <climits>
int main() {
    std::mt19937_64 rng(7);
    kvp::SlotMap m; std::unordered_map<long,long> ref;
    for (int it = 0; it < 2000000; ++it) {
        long key = (long)(rng() % 5000) - 100;
        if (rng() % 97 == 0) key = LONG_MIN;
        int op = rng() % 3;
        if (op == 0) { long v = (long)rng(); m.put(key, v); ref[key] = v; }
        else if (op == 1) { bool a = m.erase(key); bool b = ref.erase(key) > 0; if (a != b) { printf("erase mismatch\n"); return 1; } }
        else { long* p = m.find(key); auto it2 = ref.find(key); if ((p != nullptr) != (it2 != ref.end()) || (p && *p != it2->second)) { printf("find mismatch\n"); return 1; } }
        if (m.size() != ref.size()) { printf("size mismatch\n"); return 1; }
        if (it % 500000 == 0) { m.clear(); ref.clear(); }
    }
    printf("slotmap fuzz ok\n");
}
