// Exercises libkvp.so through the reference's C++ interface (include/cxx/),
// as a C++ caller of the reference would: the five TileGatingPolicy classes
// through their base-class pointer, and a KVTileManager's accounting that
// needs no device.  Built and run by tests/test_cxx_boundary.py.
//
//   cxx_boundary_check policies <n> <max_tiles> <tiles_per_frame> <total_frames> < scores
//       reads n floats (text) and prints, per policy, "name count id id ...".
//   cxx_boundary_check manager
//       prints the inline accessors of a fresh manager and the result of an
//       admission larger than the window limit (KVTM_INVALID without any
//       CUDA call).
#include "attn_kernel.h"
#include "kv_tile_manager.h"
#include "tile_gating_policy.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <vector>

static int run_policies(int n, int max_tiles, int tpf, int total_frames) {
    std::vector<float> scores((size_t)n);
    for (int i = 0; i < n; ++i)
        if (std::scanf("%f", &scores[(size_t)i]) != 1) return 2;
    std::unique_ptr<TileGatingPolicy> pols[] = {
        std::unique_ptr<TileGatingPolicy>(new NoPersistencePolicy()),
        std::unique_ptr<TileGatingPolicy>(new UniformWindowPolicy()),
        std::unique_ptr<TileGatingPolicy>(new RecencyWindowPolicy()),
        std::unique_ptr<TileGatingPolicy>(new MotionGatedPolicy()),
        std::unique_ptr<TileGatingPolicy>(new ReuseWeightedPolicy(tpf, total_frames)),
    };
    std::vector<long> ids((size_t)(max_tiles > n ? max_tiles : n) + 1);
    for (auto& p : pols) {
        int count = -1;
        p->select(scores.data(), n, max_tiles, ids.data(), &count);
        std::printf("%s %d", p->name(), count);
        for (int i = 0; i < count; ++i) std::printf(" %ld", ids[(size_t)i]);
        std::printf("\n");
    }
    return 0;
}

static int run_manager() {
    KVTileManager mgr(4096, 1024);
    std::printf("persisted_bytes %zu\n", mgr.persisted_bytes());
    std::printf("persisted_tiles %d\n", mgr.persisted_tiles());
    std::printf("arena_ptr_null %d\n", mgr.arena_device_ptr() == nullptr ? 1 : 0);
    std::printf("arena_used %zu\n", mgr.arena_used_bytes());
    std::printf("staged_bytes %zu\n", mgr.streaming_staged_bytes());
    static char host_buf[2048];
    std::printf("admit_too_large %d\n", (int)mgr.admit(7, host_buf, 2048));
    std::printf("admit_bad_args %d\n", (int)mgr.admit(-1, nullptr, 16));
    std::printf("release_unknown %d\n", mgr.release(3) ? 1 : 0);
    std::printf("is_persisted %d\n", mgr.is_persisted(7) ? 1 : 0);
    std::printf("ktile %d warps %d\n", ATTENTION_KTILE, ATTENTION_WARPS);
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 6 && std::strcmp(argv[1], "policies") == 0)
        return run_policies(std::atoi(argv[2]), std::atoi(argv[3]), std::atoi(argv[4]),
                            std::atoi(argv[5]));
    if (argc >= 2 && std::strcmp(argv[1], "manager") == 0) return run_manager();
    std::fprintf(stderr, "usage: %s policies n max tpf frames | manager\n", argv[0]);
    return 2;
}
