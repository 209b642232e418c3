// xchg_internal.cuh - the exchange object of the sharded decodes as the
// library's own code sees it: the per-rank region layout, the peer
// mappings, and the system-scope flag operations the exchanging kernels
// use. Not part of the C ABI (include/pickle_cuda.h has the opaque type).
//
// A rank's region is one cudaMalloc, mapped into every other rank's
// address space through CUDA IPC (or, for ranks driven by one process,
// used directly):
//   [0, buf_bytes)                 receive buffer
//   ready[8], done[8], epoch[8]    flags of pickle_cuda_xchg_put_dev, one word per sender
//   row_epoch[kXchgMaxRows]        this rank's call counter of each row of the fused
//                                  decode exchanges (their data words carry the epoch)
#pragma once
#include <cstddef>
#include <cstdint>

#include "pcu_common.cuh"
#include "pickle_cuda.h"

constexpr int kXchgMaxRanks = PICKLE_CUDA_XCHG_MAX_RANKS;
constexpr int kXchgMaxRows = 4096;

struct pickle_cuda_xchg {
    int rank = 0, world = 0, device = 0;
    size_t buf_bytes = 0, ready_off = 0, done_off = 0, epoch_off = 0, region_bytes = 0;
    size_t row_epoch_off = 0;
    unsigned char* region = nullptr;                 // this rank's allocation
    unsigned char* peer[kXchgMaxRanks] = {};         // mapped regions (peer[rank] = region)
    bool opened[kXchgMaxRanks] = {};
    bool ipc_mapped[kXchgMaxRanks] = {};             // opened through CUDA IPC (closed at free)
    bool broken = false;                             // a bounded wait gave up: the epochs no longer agree
    unsigned long long wait_ns = 1000000000ull;      // bound of every flag wait
    int* err_dev = nullptr;
    char last_error[256] = {0};
};

// What an exchanging kernel needs to reach every rank's region.
struct XchgPeers {
    unsigned char* base[kXchgMaxRanks];
    unsigned long long row_epoch_off;
    unsigned long long wait_ns;
    int rank, world;
};

inline XchgPeers xchg_peers(const pickle_cuda_xchg* x) {
    XchgPeers p{};
    for (int r = 0; r < x->world; ++r) p.base[r] = x->peer[r];
    p.row_epoch_off = x->row_epoch_off;
    p.wait_ns = x->wait_ns;
    p.rank = x->rank;
    p.world = x->world;
    return p;
}

PCU_DEV void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

PCU_DEV unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
