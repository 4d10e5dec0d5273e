// Shared device helpers of the Espalier B200 kernels: status codes, 16-bit float conversions, the 128-point
// Walsh-Hadamard transform in the reference's butterfly order, bounded mbarrier waits, 16-byte asynchronous copies.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/espalier_b200.h"

namespace esp {

constexpr float HAD_SCALE = 0.08838834764831845f;   // 1 / sqrt(128), the reference's float literal (dense.cu:23)

enum DType : int { F16 = ESP_DTYPE_F16, BF16 = ESP_DTYPE_BF16, F32 = ESP_DTYPE_F32 };

// Device-side error word of this translation unit: kernels that give up a bounded wait record ESP_ERR_TIMEOUT here
// and return. Each .cu file exposes its word through ESP_DEFINE_STATUS_READER; esp_device_status() reads them all.
static __device__ int g_device_status = 0;

#define ESP_DEFINE_STATUS_READER(NAME)                                                          \
    namespace esp {                                                                            \
    int status_##NAME(int reset) {                                                             \
        int v = 0;                                                                             \
        if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return -1; \
        if (reset) {                                                                           \
            const int z = 0;                                                                   \
            if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)) != cudaSuccess) return -1;  \
        }                                                                                      \
        return v;                                                                              \
    }                                                                                          \
    }

__device__ __forceinline__ void report(int code) { atomicCAS(&g_device_status, 0, code); }

// ---------------------------------------------------------------------------------------------------------------
// 4 consecutive values of a row as fp32, and back (dense.cu:56-89)
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void load4(const void* p, int dtype, size_t i, float (&v)[4]) {
    if (dtype == F32) {
        const float4 u = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
        v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
    } else if (dtype == BF16) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + i);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
}

__device__ __forceinline__ void store4(void* p, int dtype, size_t i, const float (&v)[4]) {
    if (dtype == F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
    } else if (dtype == BF16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + i) = u;
    } else {
        __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__half*>(p) + i) = u;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Hadamard-128 of one row, 4 values a lane (lane L holds elements 4L..4L+3): H4 in registers, then xor-partner stages
// 1..16 across lanes, lower lane a + b, upper lane a - b. The reference's order (dense.cu:43-54), so rotated
// activations are bit-identical to its own.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void fwht128(float (&v)[4], int lane) {
    const float a = v[0] + v[1], b = v[0] - v[1], c = v[2] + v[3], d = v[2] - v[3];
    v[0] = a + c; v[1] = b + d; v[2] = a - c; v[3] = b - d;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
            v[j] = (lane & m) ? o - v[j] : v[j] + o;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier primitives, sm_90+ PTX. Waits are bounded: after WAIT_NS of wall time the wait reports
// ESP_ERR_TIMEOUT and returns false, so no kernel can spin forever.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t WAIT_NS = 200ull * 1000 * 1000;   // a wait gives up after 0.2 s of wall time, never hangs

// Wait for the phase of `parity` to complete. Gives up after WAIT_NS (time, not polls: a suspended try_wait may sleep),
// records ESP_ERR_TIMEOUT and returns false. Once any wait of this file's kernels has timed out, a later wait gives up
// after 20 us instead, so a broken pipeline ends in about one WAIT_NS, not one a stage.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS) break;
        if (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT) return false;
    }
    report(ESP_ERR_TIMEOUT);
    return false;
}

// GPU-scope acquire load and release add (cross-CTA readiness counters).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Tagged 64-bit words (value bits in the low half, a nonzero tag in the high half): each word is written and read
// whole (single-copy atomic at GPU scope), so a reader that sees the tag sees the value, with no fence on either side.
__device__ __forceinline__ void st_relaxed_v2_u64(void* p, uint64_t a, uint64_t b) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_relaxed_v2_u64(const void* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Thread-block cluster: this CTA's rank, a barrier of every thread of the cluster (release / acquire, so shared
// memory written before it is visible to the other CTAs' reads after it), and loads from another CTA's shared memory.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 ld_cluster_f4(const void* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}

// Release/acquire fence at GPU scope. One thread executes it after a CTA barrier: the fence is cumulative over the
// writes the barrier ordered before it, so the whole CTA's stores are published without a fence in every thread.
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Split-K / last-arriver arrival: one atomic add with release and acquire semantics at GPU scope, returning the old
// value. Executed by one thread after a CTA barrier it publishes the whole CTA's earlier writes (release is cumulative
// over what the barrier ordered before it) and, for the last arriver, makes the other arrivals' writes visible; one L2
// round trip instead of fence + atomic + fence.
__device__ __forceinline__ int arrive_acq_rel(int* counter) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
    return old;
}

// 16-byte asynchronous copy global -> shared (L2 only), and the arrive-on of an mbarrier when all of this thread's
// earlier copies have landed (the arrival counts against the barrier's expected count).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// the same with a shared-window address (no generic -> shared conversion in the issuing loop)
__device__ __forceinline__ void cp_async16_sa(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory (the tensor memory accelerator, no tensor map), completing `bytes`
// on the mbarrier's transaction count. Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// Programmatic dependent launch: let the next kernel on the stream start its prologue / wait for the previous one.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace esp
