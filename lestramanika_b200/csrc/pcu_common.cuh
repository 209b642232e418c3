// pcu_common.cuh - sm_100a PTX helpers shared by the attention kernels:
// mbarriers with bounded waits, 1-D bulk (TMA) copies global -> shared,
// and the device error word.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#define PCU_DEV __device__ __forceinline__

// Device-side error codes written to the handle's error word.
enum : int {
    PCU_DEVERR_NONE = 0,
    PCU_DEVERR_FULL_WAIT = 1,    // consumer gave up waiting for a tile
    PCU_DEVERR_EMPTY_WAIT = 2,   // producer gave up waiting for a free stage
    PCU_DEVERR_DRAIN_WAIT = 3,   // copies still in flight at exit after an abort
    PCU_DEVERR_MMA_WAIT = 4,     // tensor-core completion never arrived
    PCU_DEVERR_ARG = 5,          // a device-side argument (position, slot) out of range
    PCU_DEVERR_PEER_WAIT = 6,    // another rank's flag never reached this call's epoch
};

// Every spin on an mbarrier gives up after this long and records an error
// instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000000000ull;   // 1 s

PCU_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

PCU_DEV uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

PCU_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make initialised barriers visible to the async (TMA) proxy.
PCU_DEV void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

PCU_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

PCU_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

PCU_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with `parity` to complete; false after kWaitLimitNs.
PCU_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        #pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1-D bulk copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing
// on `bar` as transaction bytes. No multicast.
PCU_DEV void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of `bytes` (multiple of 16, 16-byte aligned) from global
// memory into L2 only: no shared memory, no barrier, nothing to wait for.
// It lets a CTA keep more DRAM requests in flight than its shared-memory
// ring holds; the later bulk copy of the same bytes then hits L2.
PCU_DEV void bulk_prefetch_l2(const void* src_gmem, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}

// Programmatic dependent launch: a dependent grid waits here until its
// prerequisite grid has completed and that grid's writes are visible; the
// prerequisite lets the dependent be scheduled once all its CTAs ran this.
PCU_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
PCU_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

PCU_DEV bool tid_is_first() { return threadIdx.x == 0; }

// NeoX rotation of one float4 chunk pair (x0 = x[i..i+3], x1 = x[i+half..])
// by the table row's sin/cos (src/pickle_fast.c:1917-1924):
//   lo = c*x0 - s*x1, hi = s*x0 + c*x1,
// with the roundings fixed (one product, then one fused multiply-add), so
// every kernel that writes rotated rows writes the same bits.
PCU_DEV void rope_pair4(const float4& x0, const float4& x1, const float4& sn, const float4& cs, float4& lo,
                        float4& hi) {
    lo = make_float4(fmaf(cs.x, x0.x, -(sn.x * x1.x)), fmaf(cs.y, x0.y, -(sn.y * x1.y)),
                     fmaf(cs.z, x0.z, -(sn.z * x1.z)), fmaf(cs.w, x0.w, -(sn.w * x1.w)));
    hi = make_float4(fmaf(sn.x, x0.x, cs.x * x1.x), fmaf(sn.y, x0.y, cs.y * x1.y),
                     fmaf(sn.z, x0.z, cs.z * x1.z), fmaf(sn.w, x0.w, cs.w * x1.w));
}

// Four floats as BF16 (round to nearest even), packed for one 8-byte store.
PCU_DEV uint2 pack_bf16x4(float4 x, float scale) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(x.x * scale, x.y * scale);
    __nv_bfloat162 hi = __floats2bfloat162_rn(x.z * scale, x.w * scale);
    return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

PCU_DEV void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}
