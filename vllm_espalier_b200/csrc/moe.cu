// Grouped routed + shared expert pipeline for 1..32 tokens of one MoE layer.
//
// Reference behaviour (vllm_espalier/experts.py:231-261 routed2 and csrc/experts.cu, experts_grouped.cuh): per slot p =
// row * slots + j (the row's j-th pick; the shared expert, if any, as the last slot) with expert e = pick[p]:
//   xg/xu[p]  = fp16(H(x[row] * suh_g/u[e]) / sqrt(128))                       rot_in           experts.cu:97-115
//   g, u      = xg[p] @ W_gate[e], xu[p] @ W_up[e]  (fp32 sums)                 grouped, mats=2  experts_grouped.cuh
//   xd[p]     = fp16(H(silu(H(g) h svh_g) * H(u) h svh_u * suh_d) h)            gateup_epilogue  experts.cu:120-162
//   d         = xd[p] @ W_down[e]                                               grouped, mats=1
//   y[p]      = H(d) h svh_d (fp32); out[row] = sum_j<n_routed fma(w, y) in slot order; shared = w * y   down_combine2
// with h = 1/sqrt(128) and H the 128-point Hadamard per 128-block.
//
// B200 pipeline (4 launches after this file's kernels: route, rot_in, gate+up, down):
//   * grouped_kernel decodes, per distinct expert u (uids / members from the routing), the 8 tiles of a 128-column
//     block b at each k-tile of its k-slice, from a shared-memory stage ring filled by two producer warps with
//     16-byte cp.async (the expert's tiles and its members' rotated activation slices; gate and up units alternate, a
//     producer and a consumer group to each matrix), 16 consumer warps, one tile a warp,
//     mma.sync m16n8k16 with the weights as A (16 output columns) and up to 32 member rows as N. The codebook and width
//     are dispatched per expert matrix at run time (experts mix E2M1 1/2-bit and int5 3-bit; the shared one is int6).
//   * MODE_Z writes fp32 partial sums Z[mat][split][p][n] (the reference's `grouped` contract).
//   * MODE_GATEUP runs gate and up of block b in one CTA, splits K in S equal slices whose partials the last CTA of the
//     (expert, block) adds in slice order, then applies the SwiGLU epilogue and writes xd.
//   * MODE_DOWN writes y[p] and, when it is the last of a row's slots to finish a block (a per-(row, block) counter),
//     combines that row's slots in slot order into out / out_shared.
// Every sum is in a fixed order that depends on the shapes only, so a token's output never depends on the others.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "host.hpp"
#include "trellis.cuh"

ESP_DEFINE_STATUS_READER(moe)

namespace esp {
namespace {

constexpr int GWARPS = 16;                         // consumer warps (two groups of 8)
constexpr int GPROD = 2;                           // producer warps (units of even / odd position in a stage)
constexpr int GTHREADS = (GWARPS + GPROD) * 32;
constexpr int GUPS = 8;                            // units a stage
// Stage ring depth of an instance: as many stages as fit next to the reduction buffers in about 200 KB of dynamic
// shared memory (the static tables take the rest of the 227 KB), at most 12. Deep rings keep 20-50 KB of weights in
// flight an SM, enough to cover HBM latency with the small units of 1-3 bit experts.
__host__ __device__ constexpr int stage_words(int ntg, int kcap) { return 8 * (8 * 8 * kcap + 8 * ntg * 8); }
__host__ __device__ constexpr int red_bytes(int ntg) { return 2 * 8 * ntg * 132 * 4; }
__host__ __device__ constexpr int gstages(int ntg, int kcap) {
    return (200 * 1024 - red_bytes(ntg)) / (stage_words(ntg, kcap) * 4) < 12
               ? (200 * 1024 - red_bytes(ntg)) / (stage_words(ntg, kcap) * 4)
               : 12;
}
constexpr int GRED = 132;                          // fp32 row stride of the reduction buffers

enum Mode : int { MODE_Z = 0, MODE_GATEUP = 1, MODE_DOWN = 2 };

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }

struct GroupedParams {
    const int64_t* tp[2];          // trellis pointers a matrix slot [E]
    const int* k2[2];              // half-bits [E]
    const int* cb[2];              // kernel codebook ids [E]
    const __half* X[2];            // rotated inputs [P][K] fp16
    const int* uids;
    const int* ucount;
    const int* members;            // [maxu][maxm] row * 32 + slot, -1 padded
    int maxm, slots, K, N, P, S, mats, mode, E;
    float* Z;                      // MODE_Z: [mats][S][P][N]; MODE_GATEUP (S > 1): [2][S][P][N] partials
    int* counters;                 // MODE_GATEUP: [maxu][N/128]; MODE_DOWN: [rows][N/128]; zero, left zero
    int* work;                     // fused modes: the item counter (after the arrival counters); zero, left zero
    // MODE_GATEUP epilogue
    const __half* svh_g;           // [E][N]
    const __half* svh_u;
    const __half* suh_d;           // [E][N]
    __half* xd;                    // [P][N]
    // MODE_DOWN epilogue and combine
    const __half* svh_d;           // [E][N]
    const int* pick;               // [P]
    const float* wts;              // [P]
    float* y;                      // [P][N]
    void* out;                     // [rows][N] out_dtype
    void* out_shared;              // [rows][N] or null
    int out_dtype, n_routed;
};

// ------------------------------------------------------------------------------------------------------------------
// rot_in (experts.cu:97-115): xg/xu[p] = fp16(H(x[row] * suh[e]) h) for every slot with a valid expert. A warp per
// (slot, 128-block, matrix).
// ------------------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) rot_in_kernel(const T* __restrict__ x, long long x_stride,
                                                     const int* __restrict__ pick, const __half* __restrict__ suh0,
                                                     const __half* __restrict__ suh1, __half* __restrict__ out0,
                                                     __half* __restrict__ out1, int P, int K, int slots, int E) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int w = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nblk = K / 128;
    if (w >= P * nblk * 2) return;
    const int mat = w / (P * nblk), rem = w % (P * nblk), p = rem / nblk, blk = rem % nblk;
    const int e = pick[p];
    if (e < 0 || e >= E) return;
    const int row = p / slots;
    const int k = blk * 128 + 4 * lane;
    const __half* suh = (mat ? suh1 : suh0) + (size_t)e * K + k;
    const T* xr = x + (size_t)row * x_stride + k;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(to_f<T>(xr[j]), __half2float(suh[j]));
    fwht128(v, lane);
    __half* o = (mat ? out1 : out0) + (size_t)p * K + k;
    const __half2 a = __floats2half2_rn(v[0] * HAD_SCALE, v[1] * HAD_SCALE);
    const __half2 b = __floats2half2_rn(v[2] * HAD_SCALE, v[3] * HAD_SCALE);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(o) = u;
}

// ------------------------------------------------------------------------------------------------------------------
// The grouped decode GEMV
// ------------------------------------------------------------------------------------------------------------------
struct CtaWork {
    int e;            // expert
    int b;            // 128-column block
    int split;        // k-slice
    int mat0, nmats;  // matrix slots this CTA decodes
    int kt0, nkt;     // k-tiles of the slice
    int nm;           // members
};

// decode + MMA of the units [j0, j1) of one stage for one matrix, codebook and width fixed
template <int CB, int K, int NTG>
__device__ __forceinline__ void stage_units(const uint32_t* st, const uint32_t* xs0, int j0, int j1, int unit_w,
                                            int slice_w, int grp, int wl, int lane, int ntg, float (&acc)[2][NTG][4]) {
    const int g = lane >> 2, t = lane & 3;
    constexpr int TW = 8 * K;
    // this group's units are every other one; consecutive ones alternate between two accumulator sets (static indices,
    // so the accumulators stay in registers)
    auto mmas = [&](int jj, const uint32_t (&a)[4], float (&ac)[NTG][4]) {
        const uint32_t* xs = xs0 + jj * slice_w;
#pragma unroll
        for (int q = 0; q < NTG; ++q)
            if (q < ntg) mma16816(ac[q], a, xs[(8 * q + g) * 4 + t], xs[(8 * NTG + 8 * q + g) * 4 + t]);
    };
    // two units decoded back to back before their MMAs: no branch between the two decode chains, so they interleave
    auto pair = [&](int ja, int jb) {
        uint32_t a[4], b[4];
        decode_a<CB, K>(st + ja * unit_w + wl * TW, lane, a);
        decode_a<CB, K>(st + jb * unit_w + wl * TW, lane, b);
        mmas(ja, a, acc[0]);
        mmas(jb, b, acc[1]);
    };
    if (j0 == 0 && j1 == GUPS) {   // a whole stage (the common case): straight-line code
#pragma unroll
        for (int j2 = 0; j2 < GUPS; j2 += 4) pair(j2 + grp, j2 + grp + 2);
        return;
    }
    for (int jj = j0 + ((j0 & 1) != grp ? 1 : 0); jj < j1; jj += 4) {
        if (jj + 2 < j1) {
            pair(jj, jj + 2);
        } else {
            uint32_t a[4];
            decode_a<CB, K>(st + jj * unit_w + wl * TW, lane, a);
            mmas(jj, a, acc[0]);
        }
    }
}

template <int NTG, int KCAP>
__device__ __forceinline__ void dispatch_units(int cb, int K, const uint32_t* st, const uint32_t* xs0, int j0, int j1,
                                               int unit_w, int slice_w, int grp, int wl, int lane, int ntg,
                                               float (&acc)[2][NTG][4]) {
    switch (cb * 16 + K) {
#define ESP_GU_CASE(CB_, K_)                                                                                      \
    case CB_ * 16 + K_:                                                                                           \
        if constexpr (K_ <= KCAP) stage_units<CB_, K_, NTG>(st, xs0, j0, j1, unit_w, slice_w, grp, wl, lane, ntg, acc); \
        else report(ESP_ERR_UNSUPPORTED);                                                                         \
        break;
        ESP_FOR_EACH_CASE(ESP_GU_CASE)
#undef ESP_GU_CASE
        default: report(ESP_ERR_UNSUPPORTED); break;    // validated on the host; never a trap
    }
}

// All stages of one item for one matrix, codebook and width fixed (the one-launch layer): the (codebook, width)
// dispatch happens once an item, not once a stage. The item's first stage has been waited for by the caller.
template <int CB, int K, int NTG, int GST, int STW, int UWM, int SLW>
__device__ __forceinline__ bool item_stages(const uint32_t* smem, uint64_t* full, uint64_t* empty, int& slot, int& phase,
                                            int n, int grp, int wl, int lane, int ntg, float (&acc)[2][NTG][4]) {
    for (int i0 = 0;; i0 += GUPS) {
        if (i0 > 0 && !mbar_wait(&full[slot], phase)) return false;
        const uint32_t* st = smem + (size_t)slot * STW;
        const int m0 = min(GUPS, n - i0);
        if constexpr (CB > 0)
            if (m0 > 0) stage_units<CB, K, NTG>(st, st + GUPS * UWM, 0, m0, UWM, SLW, grp, wl, lane, ntg, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == GST) {
            slot = 0;
            phase ^= 1;
        }
        if (i0 + GUPS >= n) return true;
    }
}

template <int NTG, int KCAP, int GST, int STW, int UWM, int SLW>
__device__ __forceinline__ bool dispatch_item(int cb, int K, const uint32_t* smem, uint64_t* full, uint64_t* empty,
                                              int& slot, int& phase, int n, int grp, int wl, int lane, int ntg,
                                              float (&acc)[2][NTG][4]) {
    switch (cb * 16 + K) {
#define ESP_IT_CASE(CB_, K_)                                                                                      \
    case CB_ * 16 + K_:                                                                                           \
        if constexpr (K_ <= KCAP)                                                                                 \
            return item_stages<CB_, K_, NTG, GST, STW, UWM, SLW>(smem, full, empty, slot, phase, n, grp, wl, lane, \
                                                                 ntg, acc);                                        \
        break;
        ESP_FOR_EACH_CASE(ESP_IT_CASE)
#undef ESP_IT_CASE
        default: break;
    }
    report(ESP_ERR_UNSUPPORTED);    // validated on the host; the stages are still consumed, never a trap
    return item_stages<0, 1, NTG, GST, STW, UWM, SLW>(smem, full, empty, slot, phase, n, grp, wl, lane, ntg, acc);
}

// The gate/up epilogue of one member row's 4 columns of this lane (experts.cu:120-162, act_mode 1): sums times the
// codebook steps, H, * h * svh, silu(g) * u, * suh_d (never contracted into the butterfly), H, * h -> fp16 xd.
// The lane's 4 fp16 scales of a 128-column block (8 bytes), loaded ahead of the epilogue that needs them.
struct Scales4 {
    uint2 g, u, d;
};
__device__ __forceinline__ uint2 ld_scales4(const __half* v, int e, int N, int n0) {
    return *reinterpret_cast<const uint2*>(v + (size_t)e * N + n0);
}
__device__ __forceinline__ float scale_at(const uint2& s, int j) {
    const uint32_t w = j < 2 ? s.x : s.y;
    return __half2float(__ushort_as_half((unsigned short)((j & 1) ? (w >> 16) : (w & 0xffffu))));
}

__device__ __forceinline__ void swiglu_store(__half* xd, int N, const Scales4& sc, int n0, int pm, float cg, float cu,
                                             float (&gv)[4], float (&uv)[4], int lane) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        gv[j] *= cg;
        uv[j] *= cu;
    }
    fwht128(gv, lane);
    fwht128(uv, lane);
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float gg = gv[j] * HAD_SCALE * scale_at(sc.g, j);
        const float uu = uv[j] * HAD_SCALE * scale_at(sc.u, j);
        const float act = gg / (1.f + expf(-gg)) * uu;
        v[j] = __fmul_rn(act, scale_at(sc.d, j));
    }
    fwht128(v, lane);
    const __half2 a = __floats2half2_rn(v[0] * HAD_SCALE, v[1] * HAD_SCALE);
    const __half2 bq = __floats2half2_rn(v[2] * HAD_SCALE, v[3] * HAD_SCALE);
    uint2 uo;
    uo.x = *reinterpret_cast<const uint32_t*>(&a);
    uo.y = *reinterpret_cast<const uint32_t*>(&bq);
    *reinterpret_cast<uint2*>(xd + (size_t)pm * N + n0) = uo;
}

// Per work item descriptor, written into shared memory by the producer and read by the consumers.
struct ItemDesc {
    int it;                // the work item; -1: no more items for this CTA (an empty stage carries it)
    int e, b, split, mat0, nmats, kt0, nkt, nm;
    int cb0, K0, cb1, K1;
    int rows[32];          // slot index p of each member
};
// descriptor ring: the producer runs at most GSTAGES stages (so items) ahead; a slot is rewritten only after the
// consumers finished the item NDESC back, which needs NDESC >= GSTAGES + 2
constexpr int NDESC = 16;
constexpr int MAX_PEND = 1024;     // deferred arrivals a CTA (items a CTA x members an item)

// Work item `it` of MODE: (expert position u, block b, z); z = split (fused modes) or mat * S + split (MODE_Z).
// The fused modes hand items out dynamically (an atomic counter, from the last expert down: the shared expert, the
// widest and with the most members, starts first), MODE_Z round robin; sums never depend on which CTA runs an item.
__device__ __forceinline__ void item_coords(const GroupedParams& p, int it, int NB, int NZ, int& u, int& b, int& z) {
    u = it / (NB * NZ);
    const int r = it - u * NB * NZ;
    b = r / NZ;
    z = r - b * NZ;
}

template <int NTG, int KCAP>
__global__ void __launch_bounds__(GTHREADS, 1) grouped_kernel(const __grid_constant__ GroupedParams p) {
    constexpr int GSTAGES = gstages(NTG, KCAP);
    static_assert(GSTAGES >= 2 && GSTAGES + 2 <= NDESC, "stage ring / descriptor ring");
    constexpr int MP = 8 * NTG;
    constexpr int UNIT_WMAX = 8 * 8 * KCAP;            // words of a unit at the widest width served
    constexpr int SLICE_W = MP * 8;                    // words of a k-tile's member slice: [2][MP][8 halves]
    constexpr int STAGE_W = GUPS * (UNIT_WMAX + SLICE_W);
    extern __shared__ __align__(128) uint32_t smem[];
    float* red = reinterpret_cast<float*>(smem + (size_t)GSTAGES * STAGE_W);       // [2][MP][GRED]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * MP * GRED);
    uint64_t* empty = full + GSTAGES;
    __shared__ ItemDesc desc[NDESC];
    __shared__ int s_pend[MAX_PEND][2];      // deferred arrivals: (counter index, item or row code)
    __shared__ int s_npend;
    __shared__ int s_last[MAX_PEND];
    __shared__ int s_item[NDESC];            // producer 0 -> producer 1: the next item

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NB = p.N / 128;
    const int NZ = p.mode == MODE_Z ? p.mats * p.S : p.S;
    const int KT = p.K / 16;
    pdl_launch_dependents();
    pdl_wait();
    const int n_items = p.ucount[0] * NB * NZ;         // grid: one CTA an SM
    const bool dyn = p.work != nullptr;
    // deferred arrivals an item adds at most (the producer stops taking items before the table could overflow)
    const int pend_item = p.mode == MODE_DOWN ? p.maxm : (p.mode == MODE_GATEUP && p.S > 1 ? 1 : 0);
    if (threadIdx.x == 0) {
        for (int i = 0; i < GSTAGES; ++i) {
            mbar_init(&full[i], 32 * GPROD + 1);       // the producers' copy arrivals + the release of descriptors
            mbar_init(&empty[i], GWARPS);
        }
        s_npend = 0;
        fence_mbar_init();
    }
    // a zeroed descriptor ring: a consumer that reads a slot after a timed-out wait sees an empty item, never garbage
    for (int i = threadIdx.x; i < NDESC * (int)(sizeof(ItemDesc) / 4); i += GTHREADS)
        reinterpret_cast<int*>(desc)[i] = 0;
    __syncthreads();
    if (p.mode == MODE_DOWN && blockIdx.x == 0 && warp < GWARPS) {   // rows without a valid slot get zeros
        const int rows = p.P / p.slots;
        for (int r = warp; r < rows; r += GWARPS) {
            bool any = false;
            for (int j = 0; j < p.slots; ++j) {
                const int e2 = p.pick[r * p.slots + j];
                any |= e2 >= 0 && e2 < p.E;
            }
            if (any) continue;
            const float zero[4] = {0.f, 0.f, 0.f, 0.f};
            for (int n0 = 4 * lane; n0 < p.N; n0 += 128) {
                store4(p.out, p.out_dtype, (size_t)r * p.N + n0, zero);
                if (p.out_shared) store4(p.out_shared, p.out_dtype, (size_t)r * p.N + n0, zero);
            }
        }
    }
    if (!dyn && (int)blockIdx.x >= n_items) return;

    if (warp >= GWARPS) {   // ---------------- producers ----------------
        // Producer pw copies the units of position j = pw (mod 2) of every stage: with two matrices (gate, up units
        // alternate) that is matrix pw; with one, every other k-tile. Both compute each item's descriptor from global
        // memory; producer 0 writes it to shared memory and releases it with the item's stages.
        const int pw = warp - GWARPS;
        const uint32_t sbase = smem_addr(smem);
        int slot = 0, phase = 0, nstage = 0, di = 0, pend = 0;
        for (int k = 0;; ++k, di = (di + 1) % NDESC) {
            int it;
            if (dyn) {   // producer 0 takes the next item and hands it to producer 1 (64-thread named barrier)
                if (pw == 0 && lane == 0) {
                    int t = n_items;
                    if (pend + pend_item <= MAX_PEND) {
                        t = atomicAdd(p.work, 1);
                        if (t == n_items + (int)gridDim.x - 1) *p.work = 0;     // the last fetch of the launch
                    } else {
                        atomicAdd(p.work, 1);                                     // count the terminal fetch
                        t = n_items;
                    }
                    s_item[di] = t < n_items ? n_items - 1 - t : -1;
                }
                named_sync(2, 32 * GPROD);
                it = s_item[di];
                pend += pend_item;
            } else {
                it = blockIdx.x + k * (int)gridDim.x;
                if (it >= n_items) it = -1;
            }
            if (it < 0) {   // an empty stage tells the consumers there is nothing more
                if (pw == 0) {
                    if (lane == 0) {
                        desc[di].it = -1;
                        desc[di].nkt = 0;
                        desc[di].nmats = 0;
                        desc[di].nm = 0;
                    }
                    __syncwarp();
                }
                if (nstage >= GSTAGES && !mbar_wait(&empty[slot], phase ^ 1)) return;
                cp_async_arrive(&full[slot]);
                if (pw == 0 && lane == 0) mbar_arrive(&full[slot]);
                break;
            }
            int u, b, z;
            item_coords(p, it, NB, NZ, u, b, z);
            const int e = p.uids[u];
            const int split = p.mode == MODE_Z ? z % p.S : z;
            const int mat0 = p.mode == MODE_Z ? z / p.S : 0;
            const int nmats = p.mode == MODE_Z ? 1 : p.mats;
            const int mmB = min(mat0 + 1, p.mats - 1);
            const int code = lane < p.maxm ? p.members[u * p.maxm + lane] : -1;
            const int row = code >= 0 ? (code >> 5) * p.slots + (code & 31) : -1;
            const int nm = __popc(__ballot_sync(0xffffffffu, row >= 0));
            const int kt0 = split * KT / p.S, nkt = (split + 1) * KT / p.S - kt0;
            if (pw == 0) {
                // the descriptor slot was last read by the consumers' epilogue of item (this - NDESC), which ended
                // before they released the stage this item's first units need
                ItemDesc& d = desc[di];
                d.rows[lane] = row;
                if (lane == 0) {
                    d.it = it; d.e = e; d.b = b; d.split = split; d.mat0 = mat0; d.nmats = nmats; d.kt0 = kt0; d.nkt = nkt;
                    d.nm = nm; d.cb0 = p.cb[mat0][e]; d.K0 = p.k2[mat0][e] / 2; d.cb1 = p.cb[mmB][e];
                    d.K1 = p.k2[mmB][e] / 2;
                }
                __syncwarp();
            }
            const int n = nmats * nkt;
            // this producer's stream: matrix m, first k-tile ktA, kstep k-tiles a unit
            const int m = nmats == 2 ? mat0 + pw : mat0;
            const int kstep = nmats == 2 ? 1 : 2;
            const int ktA = kt0 + (nmats == 2 ? 0 : pw);
            const int Km = p.k2[m][e] / 2;
            const size_t kst = (size_t)(p.N / 16) * (8 * Km) * kstep;   // words between this stream's units
            const uint32_t* wp =
                reinterpret_cast<const uint32_t*>(p.tp[m][e]) + ((size_t)ktA * (p.N / 16) + (size_t)b * 8) * (8 * Km) + 4 * lane;
            const int wq = 16 * Km;                                          // 16-byte chunks a unit
            // member-slice chunks q0 = lane, q1 = lane + 32 (member q >> 1, half q & 1)
            const int r0 = __shfl_sync(0xffffffffu, row, (lane >> 1) & 31);
            const int r1 = __shfl_sync(0xffffffffu, row, ((lane + 32) >> 1) & 31);
            const bool x0v = lane < 2 * nm, x1v = lane + 32 < 2 * nm;
            const __half* xp0 = p.X[m] + (x0v ? (size_t)r0 * p.K + ktA * 16 + (lane & 1) * 8 : 0);
            const __half* xp1 = p.X[m] + (x1v ? (size_t)r1 * p.K + ktA * 16 + (lane & 1) * 8 : 0);
            const uint32_t xd0 = 4 * (GUPS * UNIT_WMAX + ((lane & 1) * MP + (lane >> 1)) * 4);
            const uint32_t xd1 = xd0 + 16 * 16;                               // member + 16
            for (int i0 = 0; i0 < n; i0 += GUPS) {
                if (nstage >= GSTAGES && !mbar_wait(&empty[slot], phase ^ 1)) return;
                const uint32_t sb = sbase + (uint32_t)slot * (STAGE_W * 4);
                const int m0 = min(GUPS, n - i0);
                for (int j = pw; j < m0; j += 2) {
                    const uint32_t du = sb + j * (UNIT_WMAX * 4) + 16 * lane;
                    for (int q = 0; q < wq - lane; q += 32) cp_async16_sa(du + 16 * q, wp + 4 * q);
                    if (x0v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd0, xp0);
                    if (x1v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd1, xp1);
                    wp += kst;
                    xp0 += 16 * kstep;
                    xp1 += 16 * kstep;
                }
                cp_async_arrive(&full[slot]);
                if (pw == 0 && lane == 0) mbar_arrive(&full[slot]);    // releases this item's descriptor with the stage
                ++nstage;
                if (++slot == GSTAGES) {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int grp = warp >> 3, wl = warp & 7;
    const int g = lane >> 2, t = lane & 3;
    constexpr int CT = GWARPS * 32;
    int slot = 0, phase = 0, di = 0;
    for (;; di = (di + 1) % NDESC) {
        float acc[2][NTG][4];      // [even/odd unit of this group][token group][4]
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2)
#pragma unroll
            for (int q = 0; q < NTG; ++q) acc[e2][q][0] = acc[e2][q][1] = acc[e2][q][2] = acc[e2][q][3] = 0.f;
        const ItemDesc* d = &desc[di];
        int nkt = 0, nmats = 0, ntg = 0, mcb = 0, mK = 0;
        int item = -1;
        Scales4 sc{};                 // the epilogue's scales, loaded with the item's first stage (latency hidden)
        for (int i0 = 0;; i0 += GUPS) {
            if (!mbar_wait(&full[slot], phase)) {   // gave up (status recorded): stop taking items
                item = -1;
                break;
            }
            if (i0 == 0) {   // the descriptor is published with the item's first stage
                item = d->it;
                nkt = d->nkt; nmats = d->nmats; ntg = (d->nm + 7) / 8;
                const bool mB = nmats == 2 && grp == 1;      // with two matrices, group = matrix
                mcb = mB ? d->cb1 : d->cb0;
                mK = mB ? d->K1 : d->K0;
                if (item >= 0) {
                    const int n0s = d->b * 128 + 4 * lane;
                    if (p.mode == MODE_DOWN) {
                        sc.d = ld_scales4(p.svh_d, d->e, p.N, n0s);
                    } else if (p.mode == MODE_GATEUP && p.S == 1) {
                        sc.g = ld_scales4(p.svh_g, d->e, p.N, n0s);
                        sc.u = ld_scales4(p.svh_u, d->e, p.N, n0s);
                        sc.d = ld_scales4(p.suh_d, d->e, p.N, n0s);
                    }
                }
            }
            const int n = nmats * nkt;
            const uint32_t* st = smem + (size_t)slot * STAGE_W;
            const int m0 = min(GUPS, n - i0);
            if (m0 > 0)
                dispatch_units<NTG, KCAP>(mcb, mK, st, st + GUPS * UNIT_WMAX, 0, m0, UNIT_WMAX, SLICE_W, grp, wl, lane,
                                          ntg, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == GSTAGES) {
                slot = 0;
                phase ^= 1;
            }
            if (i0 + GUPS >= n) break;
        }
        if (item < 0) break;   // no more items (or a wait gave up)

        // ---- the item's sums, even + odd units, into red[matrix][member][column]: with two matrices each group
        //      writes its own; with one, group 0 writes and group 1 adds ----
        const int col = wl * 16 + g;
        for (int gi = 0; gi < 2; ++gi) {
            if (gi == grp || nmats == 2) {
                const bool add = nmats == 1 && gi == 1;
                float* base = red + (size_t)(nmats == 2 ? grp : 0) * MP * GRED + col;
#pragma unroll
                for (int q = 0; q < NTG; ++q) {
                    float* rr = base + (size_t)(8 * q + 2 * t) * GRED;
                    const float v0 = acc[0][q][0] + acc[1][q][0], v1 = acc[0][q][1] + acc[1][q][1];
                    const float v2 = acc[0][q][2] + acc[1][q][2], v3 = acc[0][q][3] + acc[1][q][3];
                    if (!add) {
                        rr[0] = v0; rr[GRED] = v1; rr[8] = v2; rr[GRED + 8] = v3;
                    } else {
                        rr[0] += v0; rr[GRED] += v1; rr[8] += v2; rr[GRED + 8] += v3;
                    }
                }
            }
            named_sync(1, CT);
            if (nmats == 2) break;
        }
        const int cb0 = d->cb0, cb1 = d->cb1;
        const int b = d->b, nm = d->nm;
        const int n0 = b * 128 + 4 * lane;
        int u, bb, z;
        item_coords(p, item, NB, NZ, u, bb, z);

        if (p.mode == MODE_Z) {   // sums of the exact weights: the kernel form times its codebook step
            const float c0 = cb_step(cb0);
            for (int m = warp; m < nm; m += GWARPS) {
                float4 v = *reinterpret_cast<const float4*>(red + (size_t)m * GRED + 4 * lane);
                v.x *= c0; v.y *= c0; v.z *= c0; v.w *= c0;
                *reinterpret_cast<float4*>(p.Z + (((size_t)d->mat0 * p.S + d->split) * p.P + d->rows[m]) * p.N + n0) = v;
            }
        } else if (p.mode == MODE_GATEUP && p.S > 1) {   // slice partials; arrivals after the last item
            for (int m = warp; m < nm; m += GWARPS)
                for (int mi = 0; mi < 2; ++mi)
                    *reinterpret_cast<float4*>(p.Z + (((size_t)mi * p.S + d->split) * p.P + d->rows[m]) * p.N + n0) =
                        *reinterpret_cast<const float4*>(red + ((size_t)mi * MP + m) * GRED + 4 * lane);
            if (threadIdx.x == 0) {
                s_pend[s_npend][0] = u * NB + b;
                s_pend[s_npend][1] = item;
                ++s_npend;
            }
        } else if (p.mode == MODE_GATEUP) {   // whole K in this item: the epilogue now
            for (int m = warp; m < nm; m += GWARPS) {
                const float4 a = *reinterpret_cast<const float4*>(red + (size_t)m * GRED + 4 * lane);
                const float4 c4 = *reinterpret_cast<const float4*>(red + ((size_t)MP + m) * GRED + 4 * lane);
                float gv[4] = {a.x, a.y, a.z, a.w}, uv[4] = {c4.x, c4.y, c4.z, c4.w};
                swiglu_store(p.xd, p.N, sc, n0, d->rows[m], cb_step(cb0), cb_step(cb1), gv, uv, lane);
            }
        } else {   // MODE_DOWN: y for this block; row arrivals after the last item
            const float cd = cb_step(cb0);

            for (int m = warp; m < nm; m += GWARPS) {
                const float4 a = *reinterpret_cast<const float4*>(red + (size_t)m * GRED + 4 * lane);
                float v[4] = {a.x * cd, a.y * cd, a.z * cd, a.w * cd};
                fwht128(v, lane);
                float4 o;
                o.x = v[0] * HAD_SCALE * scale_at(sc.d, 0);
                o.y = v[1] * HAD_SCALE * scale_at(sc.d, 1);
                o.z = v[2] * HAD_SCALE * scale_at(sc.d, 2);
                o.w = v[3] * HAD_SCALE * scale_at(sc.d, 3);
                *reinterpret_cast<float4*>(p.y + (size_t)d->rows[m] * p.N + n0) = o;
            }
            if (threadIdx.x < nm) {
                const int r = d->rows[threadIdx.x] / p.slots;
                s_pend[s_npend + threadIdx.x][0] = r * NB + b;
                s_pend[s_npend + threadIdx.x][1] = r * 256 + b;
            }
            named_sync(1, CT);
            if (threadIdx.x == 0) s_npend += nm;
        }
        named_sync(1, CT);   // red and the descriptor are free for the next item
    }

    // ---------------- deferred arrivals: the last arriver finishes ----------------
    named_sync(1, CT);
    const int np = s_npend;
    if (np == 0) return;
    for (int i = threadIdx.x; i < np; i += CT) {
        int target;
        if (p.mode == MODE_GATEUP) {
            target = p.S;
        } else {
            const int r = s_pend[i][1] >> 8;
            target = 0;
            for (int j = 0; j < p.slots; ++j) {
                const int e2 = p.pick[r * p.slots + j];
                target += e2 >= 0 && e2 < p.E;
            }
        }
        s_last[i] = arrive_acq_rel(&p.counters[s_pend[i][0]]) == target - 1;
    }
    named_sync(1, CT);
    for (int pi = 0; pi < np; ++pi) {
        if (!s_last[pi]) continue;
        if (p.mode == MODE_GATEUP) {   // add the S slices in order, then the SwiGLU epilogue
            int u, b, z;
            item_coords(p, s_pend[pi][1], NB, NZ, u, b, z);
            const int e = p.uids[u];
            const float cg = cb_step(p.cb[0][e]), cu = cb_step(p.cb[1 % p.mats][e]);
            const int n0 = b * 128 + 4 * lane;
            const Scales4 dsc{ld_scales4(p.svh_g, e, p.N, n0), ld_scales4(p.svh_u, e, p.N, n0),
                              ld_scales4(p.suh_d, e, p.N, n0)};   // issued with the partial sums' loads
            for (int m = warp; m < p.maxm; m += GWARPS) {
                const int code = p.members[u * p.maxm + m];
                if (code < 0) continue;
                const int pm = (code >> 5) * p.slots + (code & 31);
                float4 sg = make_float4(0.f, 0.f, 0.f, 0.f), su = sg;
                for (int s2 = 0; s2 < p.S; ++s2) {
                    const float4 a = __ldcg(reinterpret_cast<const float4*>(p.Z + ((size_t)s2 * p.P + pm) * p.N + n0));
                    const float4 c4 = __ldcg(reinterpret_cast<const float4*>(p.Z + (((size_t)p.S + s2) * p.P + pm) * p.N + n0));
                    sg.x += a.x; sg.y += a.y; sg.z += a.z; sg.w += a.w;
                    su.x += c4.x; su.y += c4.y; su.z += c4.z; su.w += c4.w;
                }
                float gv[4] = {sg.x, sg.y, sg.z, sg.w}, uv[4] = {su.x, su.y, su.z, su.w};
                swiglu_store(p.xd, p.N, dsc, n0, pm, cg, cu, gv, uv, lane);
            }
            if (threadIdx.x == 0) p.counters[s_pend[pi][0]] = 0;
        } else {                        // MODE_DOWN: combine the row's slots in slot order
            const int r = s_pend[pi][1] >> 8, b = s_pend[pi][1] & 255;
            if (warp != pi % GWARPS) continue;
            const int n0 = b * 128 + 4 * lane;
            float acc4[4] = {0.f, 0.f, 0.f, 0.f};
            for (int j = 0; j < p.n_routed; ++j) {
                const int q = r * p.slots + j;
                const int e2 = p.pick[q];
                if (e2 < 0 || e2 >= p.E) continue;
                const float wq = p.wts[q];
                const float4 yv = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)q * p.N + n0));
                acc4[0] = fmaf(wq, yv.x, acc4[0]);
                acc4[1] = fmaf(wq, yv.y, acc4[1]);
                acc4[2] = fmaf(wq, yv.z, acc4[2]);
                acc4[3] = fmaf(wq, yv.w, acc4[3]);
            }
            store4(p.out, p.out_dtype, (size_t)r * p.N + n0, acc4);
            if (p.out_shared && p.n_routed < p.slots) {
                const int q = r * p.slots + p.n_routed;
                const int e2 = p.pick[q];
                float sv[4] = {0.f, 0.f, 0.f, 0.f};
                if (e2 >= 0 && e2 < p.E) {
                    const float wq = p.wts[q];
                    const float4 yv = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)q * p.N + n0));
                    sv[0] = wq * yv.x; sv[1] = wq * yv.y; sv[2] = wq * yv.z; sv[3] = wq * yv.w;
                }
                store4(p.out_shared, p.out_dtype, (size_t)r * p.N + n0, sv);
            }
            if (lane == 0) p.counters[s_pend[pi][0]] = 0;
        }
    }
}

// ------------------------------------------------------------------------------------------------------------------
// The fused expert layer: gate/up + SwiGLU and down + combine in one persistent launch.
//
// One work counter hands out every gate/up item (expert entry u, 128-column block of I, k-slice), then every down
// item (entry u, 128-column block of D), both from the last entry down. A down item's producers wait (bounded, acquire)
// until its entry's gate/up blocks have all been finished (ready[u] == I / 128) before copying its xd slices. A
// finisher warp takes the arrivals off the consumers: the last of a block's S slices to arrive adds the slices in
// order and runs the SwiGLU into xd, then releases ready[u]; the last of a row's slots to finish a down block combines
// the row in slot order. No deadlock: a waiting producer waits only for items handed out before its own, which CTAs
// already hold and finish without waiting on anything later. Sums and orders are those of the two-launch path, so the
// outputs are the same bits.
// ------------------------------------------------------------------------------------------------------------------
struct LayerParams {
    const int* uids;
    const int* ucount;
    const int* members;            // [maxu][maxm] row * 32 + slot, -1 padded
    int maxm, maxu, slots, rows, E, n_routed;
    // gate / up: D -> I (rotated inputs xg / xu [P][D])
    const int64_t* tp[3];          // trellis pointer tables: gate, up, down [E]
    const int* k2[3];
    const int* cb[3];
    const __half* xg;
    const __half* xu;
    int D, I, S;
    const __half* svh_g;
    const __half* svh_u;
    const __half* suh_d;
    float* Z;                      // [2][S][P][I] slice partials (S > 1)
    __half* xd;                    // [P][I]
    // down: I -> D
    const __half* svh_d;
    const int* pick;               // [P]
    const float* wts;              // [P]
    float* y;                      // [P][D]
    void* out;
    void* out_shared;
    int out_dtype;
    // counters, zero on entry and left zero: slice arrivals [maxu][I/128], row arrivals [rows][D/128], the work
    // counter, entry readiness [maxu], CTA exits
    int* cnt_gu;
    int* cnt_d;
    int* work;
    int* ready;
    int* exits;
    // expert parallel (ep_world > 0): the y row of slot q = (home rank h, row r, slot j) of the received rows goes
    // straight into h's inbox [R][slots][D] (a peer store), and the last CTA out releases every home's flag for this
    // rank (epoch + 1); the rows' combine then runs on their home ranks
    float* ep_y[8];
    int* ep_flag[8];
    const int* ep_epoch;
    int ep_world, ep_rank, ep_R;
};

struct FinEntry {
    int kind, u, b;                // kind 0: gate/up block (u, b) stored; 1: down block (u, b) stored; 2: no more
    int e, nm;                     // the entry's expert and member count
    float c0, c1;                  // codebook steps (gate, up)
};
// Warm the L2 with data of this layer that is not the previous kernel's output, while that kernel still runs (before
// the launch wait): the expert tables (CTA 0, 128-byte lines) and the three matrices of the last table entry, which is
// the shared expert whenever the layer has one (every call uses it; otherwise a routed expert, harmlessly), a slice a
// CTA by one bulk L2 prefetch each. Every layer has tables and experts of its own, so both would be DRAM misses.
__device__ __forceinline__ void prefetch_line_l2(const void* a) { asm volatile("prefetch.global.L2 [%0];" ::"l"(a)); }
__device__ __forceinline__ void bulk_prefetch_l2(const void* a, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(bytes) : "memory");
}

template <typename LP>
__device__ __forceinline__ void layer_prefetch(const LP& p, int threads) {
    if (blockIdx.x == 0) {
        const int l8 = (p.E * 8 + 127) / 128, l4 = (p.E * 4 + 127) / 128, per = l8 + 2 * l4;
        for (int i = threadIdx.x; i < 3 * per; i += threads) {
            const int t = i / per, j = i % per;
            const char* a = j < l8 ? reinterpret_cast<const char*>(p.tp[t]) + 128 * j
                          : j < l8 + l4 ? reinterpret_cast<const char*>(p.k2[t]) + 128 * (j - l8)
                                        : reinterpret_cast<const char*>(p.cb[t]) + 128 * (j - l8 - l4);
            prefetch_line_l2(a);
        }
    }
    if (threadIdx.x == 0) {
        const int e = p.E - 1;
        for (int t = 0; t < 3; ++t) {
            const size_t bytes = (size_t)p.D * p.I * (p.k2[t][e] / 2) / 8;   // a multiple of 16 (D, I multiples of 128)
            const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) / 16 * 16;
            const size_t off = (size_t)blockIdx.x * per;
            if (off < bytes)
                bulk_prefetch_l2(reinterpret_cast<const char*>(p.tp[t][e]) + off, (uint32_t)min(per, bytes - off));
        }
    }
}

constexpr int FQ = 32;                             // finisher queue entries
constexpr int LMAXP = 32 * 32;                     // slots a call (32 rows x 32 slots at most)
constexpr int LWARPS = GWARPS + GPROD + 1;         // + the finisher warp
constexpr int LTHREADS = LWARPS * 32;

__device__ __forceinline__ bool wait_ready(const int* ready, int need) {
    if (ld_acquire_gpu(ready) >= need) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        for (int i = 0; i < 32; ++i) {
            __nanosleep(64);
            if (ld_acquire_gpu(ready) >= need) return true;
        }
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS) break;
        if (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT) return false;
    }
    report(ESP_ERR_TIMEOUT);
    return false;
}

// Spin on a shared-memory word until it passes `v` (bounded by time like the mbarrier waits).
__device__ __forceinline__ bool wait_smem_gt(const volatile int* w, int v) {
    if (*w > v) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        for (int i = 0; i < 64; ++i) {
            __nanosleep(32);
            if (*w > v) return true;
        }
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS) break;
        if (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT) return false;
    }
    report(ESP_ERR_TIMEOUT);
    return false;
}

// The layer kernel's readiness wait on its own: one thread waits until *flag >= need (bounded by time; on giving up
// ESP_ERR_TIMEOUT is recorded in the status word) and writes 1 (reached) or 0 (gave up) to *result. It lets a test run
// the timeout path on a flag that nothing sets and check that the host reads the status and the context stays usable.
__global__ void wait_flag_kernel(const int* flag, int need, int* result) {
    if (threadIdx.x == 0) *result = wait_ready(flag, need) ? 1 : 0;
}

template <int NTG, int KCAP>
__global__ void __launch_bounds__(LTHREADS, 1) layer_kernel(const __grid_constant__ LayerParams p) {
    constexpr int GSTAGES = gstages(NTG, KCAP);
    static_assert(GSTAGES >= 2 && GSTAGES + 2 <= NDESC, "stage ring / descriptor ring");
    constexpr int MP = 8 * NTG;
    constexpr int UNIT_WMAX = 8 * 8 * KCAP;
    constexpr int SLICE_W = MP * 8;
    constexpr int STAGE_W = GUPS * (UNIT_WMAX + SLICE_W);
    extern __shared__ __align__(128) uint32_t smem[];
    float* red = reinterpret_cast<float*>(smem + (size_t)GSTAGES * STAGE_W);       // [2][MP][GRED]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * MP * GRED);
    uint64_t* empty = full + GSTAGES;
    __shared__ ItemDesc desc[NDESC];
    __shared__ int s_item[NDESC];
    __shared__ FinEntry s_q[FQ];
    __shared__ int s_qrows[FQ][32];                // each queued item's member slots (row * slots + slot)
    __shared__ int s_qtail, s_qhead;
    __shared__ float s_w[LMAXP];                   // the finisher's copies of the call's weights,
    __shared__ unsigned char s_ok[LMAXP];          // which slots are valid,
    __shared__ int s_tgt[32];                      // and each row's valid slot count

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NBg = p.I / 128, NBd = p.D / 128;
    const int KTg = p.D / 16, KTd = p.I / 16;
    const int P = p.rows * p.slots;
    layer_prefetch(p, LTHREADS);
    pdl_launch_dependents();
    pdl_wait();
    const int nu = p.ucount[0];
    const int n_gu = nu * NBg * p.S, n_items = n_gu + nu * NBd;
    if (threadIdx.x == 0) {
        for (int i = 0; i < GSTAGES; ++i) {
            mbar_init(&full[i], 32 * GPROD + 1);
            mbar_init(&empty[i], GWARPS);
        }
        s_qtail = 0;
        s_qhead = 0;
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < NDESC * (int)(sizeof(ItemDesc) / 4); i += LTHREADS)
        reinterpret_cast<int*>(desc)[i] = 0;
    __syncthreads();
    if (blockIdx.x == 0 && warp < GWARPS) {   // rows without a valid slot get zeros
        for (int r = warp; r < p.rows; r += GWARPS) {
            bool any = false;
            for (int j = 0; j < p.slots; ++j) {
                const int e2 = p.pick[r * p.slots + j];
                any |= e2 >= 0 && e2 < p.E;
            }
            if (any) continue;
            const float zero[4] = {0.f, 0.f, 0.f, 0.f};
            for (int n0 = 4 * lane; n0 < p.D; n0 += 128) {
                store4(p.out, p.out_dtype, (size_t)r * p.D + n0, zero);
                if (p.out_shared) store4(p.out_shared, p.out_dtype, (size_t)r * p.D + n0, zero);
            }
        }
    }

    if (warp >= GWARPS && warp < GWARPS + GPROD) {   // ---------------- producers ----------------
        const int pw = warp - GWARPS;
        const uint32_t sbase = smem_addr(smem);
        int slot = 0, phase = 0, nstage = 0, di = 0;
        bool first = true;
        for (;; di = (di + 1) % NDESC) {
            if (pw == 0 && lane == 0) {
                // a CTA's first item is its own index (no atomic on the critical path); the rest come from the
                // counter, offset by the grid. Every CTA with a first item makes exactly one failing fetch, so the
                // fetches number n_items and the one that returns n_items - 1 is the launch's last: it resets.
                int t = blockIdx.x;
                if (!first) {
                    const int c = atomicAdd(p.work, 1);
                    if (c == n_items - 1) *p.work = 0;
                    t = c + (int)gridDim.x;
                }
                first = false;
                s_item[di] = t < n_items ? t : -1;
            }
            named_sync(2, 32 * GPROD);
            const int t = s_item[di];
            if (t < 0) {   // an empty stage tells the consumers there is nothing more
                if (pw == 0) {
                    if (lane == 0) {
                        desc[di].it = -1;
                        desc[di].nkt = 0;
                        desc[di].nmats = 0;
                        desc[di].nm = 0;
                    }
                    __syncwarp();
                }
                if (nstage >= GSTAGES && !mbar_wait(&empty[slot], phase ^ 1)) return;
                cp_async_arrive(&full[slot]);
                if (pw == 0 && lane == 0) mbar_arrive(&full[slot]);
                break;
            }
            const bool down = t >= n_gu;
            int u, b, split;
            if (!down) {
                const int it = n_gu - 1 - t;
                u = it / (NBg * p.S);
                const int r = it - u * NBg * p.S;
                b = r / p.S;
                split = r - b * p.S;
            } else {
                const int it = n_items - 1 - t;
                u = it / NBd;
                b = it - u * NBd;
                split = 0;
            }
            const int e = p.uids[u];
            const int code = lane < p.maxm ? p.members[u * p.maxm + lane] : -1;
            const int row = code >= 0 ? (code >> 5) * p.slots + (code & 31) : -1;
            const int nm = __popc(__ballot_sync(0xffffffffu, row >= 0));
            const int K = down ? p.I : p.D, N = down ? p.D : p.I, KT = down ? KTd : KTg;
            const int S = down ? 1 : p.S;
            const int nmats = down ? 1 : 2;
            const int kt0 = split * KT / S, nkt = (split + 1) * KT / S - kt0;
            const int ta = down ? 2 : 0, tb = down ? 2 : 1;
            if (pw == 0) {
                ItemDesc& d = desc[di];
                d.rows[lane] = row;
                if (lane == 0) {
                    d.it = t; d.e = e; d.b = b; d.split = split; d.mat0 = down; d.nmats = nmats; d.kt0 = kt0;
                    d.nkt = nkt; d.nm = nm; d.cb0 = p.cb[ta][e]; d.K0 = p.k2[ta][e] / 2; d.cb1 = p.cb[tb][e];
                    d.K1 = p.k2[tb][e] / 2;
                }
                __syncwarp();
            }
            const int n = nmats * nkt;
            const int m = nmats == 2 ? pw : 0;
            const int tsel = down ? 2 : m;
            const int kstep = nmats == 2 ? 1 : 2;
            const int ktA = kt0 + (nmats == 2 ? 0 : pw);
            const int Km = p.k2[tsel][e] / 2;
            const size_t kst = (size_t)(N / 16) * (8 * Km) * kstep;
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(p.tp[tsel][e]) +
                                 ((size_t)ktA * (N / 16) + (size_t)b * 8) * (8 * Km) + 4 * lane;
            const int wq = 16 * Km;
            const __half* X = down ? p.xd : (m == 0 ? p.xg : p.xu);
            const int r0 = __shfl_sync(0xffffffffu, row, (lane >> 1) & 31);
            const int r1 = __shfl_sync(0xffffffffu, row, ((lane + 32) >> 1) & 31);
            const bool x0v = lane < 2 * nm, x1v = lane + 32 < 2 * nm;
            const __half* xp0 = X + (x0v ? (size_t)r0 * K + ktA * 16 + (lane & 1) * 8 : 0);
            const __half* xp1 = X + (x1v ? (size_t)r1 * K + ktA * 16 + (lane & 1) * 8 : 0);
            const uint32_t xd0 = 4 * (GUPS * UNIT_WMAX + ((lane & 1) * MP + (lane >> 1)) * 4);
            const uint32_t xd1 = xd0 + 16 * 16;
            int i0 = 0;
            if (down) {
                // the weights do not depend on the gate/up results: the first stages (as many as the ring holds) get
                // theirs before the entry's readiness wait (every gate/up block's SwiGLU done), their xd slices after
                int ps = slot;
                for (int npf = 0; i0 < n && npf < GSTAGES; i0 += GUPS, ++npf) {
                    if (nstage >= GSTAGES && !mbar_wait(&empty[slot], phase ^ 1)) return;
                    const uint32_t sb = sbase + (uint32_t)slot * (STAGE_W * 4);
                    const int m0 = min(GUPS, n - i0);
                    for (int j = pw; j < m0; j += 2) {
                        const uint32_t du = sb + j * (UNIT_WMAX * 4) + 16 * lane;
                        for (int q = 0; q < wq - lane; q += 32) cp_async16_sa(du + 16 * q, wp + 4 * q);
                        wp += kst;
                    }
                    ++nstage;
                    if (++slot == GSTAGES) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
                if (lane == 0 && !wait_ready(p.ready + u, NBg)) {
                    // gave up (status recorded): the item runs on whatever xd holds
                }
                __syncwarp();
                for (int i1 = 0; i1 < i0; i1 += GUPS) {
                    const uint32_t sb = sbase + (uint32_t)ps * (STAGE_W * 4);
                    const int m0 = min(GUPS, n - i1);
                    for (int j = pw; j < m0; j += 2) {
                        if (x0v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd0, xp0);
                        if (x1v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd1, xp1);
                        xp0 += 16 * kstep;
                        xp1 += 16 * kstep;
                    }
                    cp_async_arrive(&full[ps]);
                    if (pw == 0 && lane == 0) mbar_arrive(&full[ps]);
                    if (++ps == GSTAGES) ps = 0;
                }
            }
            for (; i0 < n; i0 += GUPS) {
                if (nstage >= GSTAGES && !mbar_wait(&empty[slot], phase ^ 1)) return;
                const uint32_t sb = sbase + (uint32_t)slot * (STAGE_W * 4);
                const int m0 = min(GUPS, n - i0);
                for (int j = pw; j < m0; j += 2) {
                    const uint32_t du = sb + j * (UNIT_WMAX * 4) + 16 * lane;
                    for (int q = 0; q < wq - lane; q += 32) cp_async16_sa(du + 16 * q, wp + 4 * q);
                    if (x0v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd0, xp0);
                    if (x1v) cp_async16_sa(sb + j * (SLICE_W * 4) + xd1, xp1);
                    wp += kst;
                    xp0 += 16 * kstep;
                    xp1 += 16 * kstep;
                }
                cp_async_arrive(&full[slot]);
                if (pw == 0 && lane == 0) mbar_arrive(&full[slot]);
                ++nstage;
                if (++slot == GSTAGES) {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
        return;
    }

    if (warp == GWARPS + GPROD) {   // ---------------- finisher ----------------
        // everything but the arrivals and the partial sums comes from shared memory: the queue entry (expert, steps,
        // member slots) and the call's picks / weights / per-row counts, loaded here while the first items decode
        for (int q = lane; q < P; q += 32) {
            const int e2 = p.pick[q];
            s_ok[q] = e2 >= 0 && e2 < p.E;
            s_w[q] = p.wts[q];
        }
        __syncwarp();
        for (int r = lane; r < p.rows; r += 32) {
            int c = 0;
            for (int j = 0; j < p.slots; ++j) c += s_ok[r * p.slots + j];
            s_tgt[r] = c;
        }
        __syncwarp();
        int head = 0;
        for (;;) {
            if (!wait_smem_gt(&s_qtail, head)) break;
            __threadfence_block();
            const FinEntry f = s_q[head % FQ];
            const int* qrows = s_qrows[head % FQ];
            if (f.kind == 2) break;
            const int n0 = f.b * 128 + 4 * lane;
            if (f.kind == 0) {   // a gate/up block's slice: the last of the S adds them and runs the SwiGLU
                const Scales4 sc{ld_scales4(p.svh_g, f.e, p.I, n0), ld_scales4(p.svh_u, f.e, p.I, n0),
                                 ld_scales4(p.suh_d, f.e, p.I, n0)};   // constant data: loaded ahead of the arrival
                int last = 0;
                if (lane == 0) last = arrive_acq_rel(&p.cnt_gu[f.u * NBg + f.b]) == p.S - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                __syncwarp();
                if (last) {
                    for (int m = 0; m < f.nm; ++m) {
                        const int pm = qrows[m];
                        float4 sg = make_float4(0.f, 0.f, 0.f, 0.f), su = sg;
                        for (int s0 = 0; s0 < p.S; s0 += 2) {   // two slices' loads in flight, added in order
                            float4 a[2], c4[2];
#pragma unroll
                            for (int q = 0; q < 2; ++q)
                                if (s0 + q < p.S) {
                                    a[q] = __ldcg(reinterpret_cast<const float4*>(p.Z + ((size_t)(s0 + q) * P + pm) * p.I + n0));
                                    c4[q] = __ldcg(reinterpret_cast<const float4*>(
                                        p.Z + (((size_t)p.S + s0 + q) * P + pm) * p.I + n0));
                                }
#pragma unroll
                            for (int q = 0; q < 2; ++q)
                                if (s0 + q < p.S) {
                                    sg.x += a[q].x; sg.y += a[q].y; sg.z += a[q].z; sg.w += a[q].w;
                                    su.x += c4[q].x; su.y += c4[q].y; su.z += c4[q].z; su.w += c4[q].w;
                                }
                        }
                        float gv[4] = {sg.x, sg.y, sg.z, sg.w}, uv[4] = {su.x, su.y, su.z, su.w};
                        swiglu_store(p.xd, p.I, sc, n0, pm, f.c0, f.c1, gv, uv, lane);
                    }
                    __syncwarp();
                    if (lane == 0) {
                        p.cnt_gu[f.u * NBg + f.b] = 0;
                        red_release_gpu_add(p.ready + f.u, 1);
                    }
                }
            } else {             // a down block of the entry's members: the last of a row's slots combines the row
                int r = -1, last = 0;
                if (lane < f.nm) {
                    r = qrows[lane] / p.slots;
                    last = arrive_acq_rel(&p.cnt_d[r * NBd + f.b]) == s_tgt[r] - 1;
                }
                unsigned lastm = __ballot_sync(0xffffffffu, last);
                __syncwarp();
                while (lastm) {
                    const int src = __ffs(lastm) - 1;
                    lastm &= lastm - 1;
                    const int rr = __shfl_sync(0xffffffffu, r, src);
                    const int q0 = rr * p.slots;
                    const bool shs = p.out_shared && p.n_routed < p.slots && s_ok[q0 + p.n_routed];
                    float4 ysh = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (shs) ysh = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)(q0 + p.n_routed) * p.D + n0));
                    float acc4[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int j0 = 0; j0 < p.n_routed; j0 += 8) {   // eight slots' loads in flight, summed in order
                        float4 yv[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (j0 + q < p.n_routed && s_ok[q0 + j0 + q])
                                yv[q] = __ldcg(reinterpret_cast<const float4*>(p.y + (size_t)(q0 + j0 + q) * p.D + n0));
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (j0 + q < p.n_routed && s_ok[q0 + j0 + q]) {
                                const float wq = s_w[q0 + j0 + q];
                                acc4[0] = fmaf(wq, yv[q].x, acc4[0]);
                                acc4[1] = fmaf(wq, yv[q].y, acc4[1]);
                                acc4[2] = fmaf(wq, yv[q].z, acc4[2]);
                                acc4[3] = fmaf(wq, yv[q].w, acc4[3]);
                            }
                    }
                    store4(p.out, p.out_dtype, (size_t)rr * p.D + n0, acc4);
                    if (p.out_shared && p.n_routed < p.slots) {
                        float sv[4] = {0.f, 0.f, 0.f, 0.f};
                        if (shs) {
                            const float wq = s_w[q0 + p.n_routed];
                            sv[0] = wq * ysh.x; sv[1] = wq * ysh.y; sv[2] = wq * ysh.z; sv[3] = wq * ysh.w;
                        }
                        store4(p.out_shared, p.out_dtype, (size_t)rr * p.D + n0, sv);
                    }
                    if (lane == 0) p.cnt_d[rr * NBd + f.b] = 0;
                }
            }
            ++head;
            __syncwarp();
            if (lane == 0) *reinterpret_cast<volatile int*>(&s_qhead) = head;
        }
    } else {                         // ---------------- consumers ----------------
        const int grp = warp >> 3, wl = warp & 7;
        const int g = lane >> 2, t = lane & 3;
        constexpr int CT = GWARPS * 32;
        int slot = 0, phase = 0, di = 0;
        auto enqueue = [&](int kind, int u, const ItemDesc* d) {   // warp 0
            const int tail = *reinterpret_cast<volatile int*>(&s_qtail);
            int room = 1;
            if (lane == 0) room = wait_smem_gt(&s_qhead, tail - FQ);   // the finisher frees entries
            if (!__shfl_sync(0xffffffffu, room, 0)) return;
            if (d) s_qrows[tail % FQ][lane] = d->rows[lane];
            if (lane == 0)
                s_q[tail % FQ] = d ? FinEntry{kind, u, d->b, d->e, d->nm, cb_step(d->cb0), cb_step(d->cb1)}
                                   : FinEntry{kind, 0, 0, 0, 0, 0.f, 0.f};
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                *reinterpret_cast<volatile int*>(&s_qtail) = tail + 1;
            }
        };
        for (;; di = (di + 1) % NDESC) {
            float acc[2][NTG][4];
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2)
#pragma unroll
                for (int q = 0; q < NTG; ++q) acc[e2][q][0] = acc[e2][q][1] = acc[e2][q][2] = acc[e2][q][3] = 0.f;
            const ItemDesc* d = &desc[di];
            int nkt = 0, nmats = 0, ntg = 0, mcb = 0, mK = 0, item = -1;
            Scales4 sc{};
            if (!mbar_wait(&full[slot], phase)) break;   // the item's first stage (or the end marker)
            item = d->it;
            if (item < 0) {                               // the end marker: release its stage and leave
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                break;
            }
            nkt = d->nkt; nmats = d->nmats; ntg = (d->nm + 7) / 8;
            {
                const bool mB = nmats == 2 && grp == 1;
                mcb = mB ? d->cb1 : d->cb0;
                mK = mB ? d->K1 : d->K0;
                const int n0s = d->b * 128 + 4 * lane;
                if (item >= n_gu) {
                    sc.d = ld_scales4(p.svh_d, d->e, p.D, n0s);
                } else if (p.S == 1) {
                    sc.g = ld_scales4(p.svh_g, d->e, p.I, n0s);
                    sc.u = ld_scales4(p.svh_u, d->e, p.I, n0s);
                    sc.d = ld_scales4(p.suh_d, d->e, p.I, n0s);
                }
            }
            if (!dispatch_item<NTG, KCAP, GSTAGES, STAGE_W, UNIT_WMAX, SLICE_W>(mcb, mK, smem, full, empty, slot, phase,
                                                                                 nmats * nkt, grp, wl, lane, ntg, acc))
                break;

            const int col = wl * 16 + g;
            for (int gi = 0; gi < 2; ++gi) {
                if (gi == grp || nmats == 2) {
                    const bool add = nmats == 1 && gi == 1;
                    float* base = red + (size_t)(nmats == 2 ? grp : 0) * MP * GRED + col;
#pragma unroll
                    for (int q = 0; q < NTG; ++q) {
                        float* rr = base + (size_t)(8 * q + 2 * t) * GRED;
                        const float v0 = acc[0][q][0] + acc[1][q][0], v1 = acc[0][q][1] + acc[1][q][1];
                        const float v2 = acc[0][q][2] + acc[1][q][2], v3 = acc[0][q][3] + acc[1][q][3];
                        if (!add) {
                            rr[0] = v0; rr[GRED] = v1; rr[8] = v2; rr[GRED + 8] = v3;
                        } else {
                            rr[0] += v0; rr[GRED] += v1; rr[8] += v2; rr[GRED + 8] += v3;
                        }
                    }
                }
                named_sync(1, CT);
                if (nmats == 2) break;
            }
            const int cb0 = d->cb0, cb1 = d->cb1, b = d->b, nm = d->nm;
            const bool down = item >= n_gu;
            const int u = down ? (n_items - 1 - item) / NBd : (n_gu - 1 - item) / (NBg * p.S);
            if (!down && p.S > 1) {            // slice partials for the finisher
                const int n0 = b * 128 + 4 * lane;
                for (int m = warp; m < nm; m += GWARPS)
                    for (int mi = 0; mi < 2; ++mi)
                        *reinterpret_cast<float4*>(p.Z + (((size_t)mi * p.S + d->split) * P + d->rows[m]) * p.I + n0) =
                            *reinterpret_cast<const float4*>(red + ((size_t)mi * MP + m) * GRED + 4 * lane);
                named_sync(1, CT);
                if (warp == 0) enqueue(0, u, d);
            } else if (!down) {                // the whole of K in this item: the SwiGLU now, then the entry's release
                const int n0 = b * 128 + 4 * lane;
                for (int m = warp; m < nm; m += GWARPS) {
                    const float4 a = *reinterpret_cast<const float4*>(red + (size_t)m * GRED + 4 * lane);
                    const float4 c4 = *reinterpret_cast<const float4*>(red + ((size_t)MP + m) * GRED + 4 * lane);
                    float gv[4] = {a.x, a.y, a.z, a.w}, uv[4] = {c4.x, c4.y, c4.z, c4.w};
                    swiglu_store(p.xd, p.I, sc, n0, d->rows[m], cb_step(cb0), cb_step(cb1), gv, uv, lane);
                }
                named_sync(1, CT);
                if (threadIdx.x == 0) red_release_gpu_add(p.ready + u, 1);
            } else {                           // y for this block, then the rows' arrivals through the finisher
                const float cd = cb_step(cb0);
                const int n0 = b * 128 + 4 * lane;
                for (int m = warp; m < nm; m += GWARPS) {
                    const float4 a = *reinterpret_cast<const float4*>(red + (size_t)m * GRED + 4 * lane);
                    float v[4] = {a.x * cd, a.y * cd, a.z * cd, a.w * cd};
                    fwht128(v, lane);
                    float4 o;
                    o.x = v[0] * HAD_SCALE * scale_at(sc.d, 0);
                    o.y = v[1] * HAD_SCALE * scale_at(sc.d, 1);
                    o.z = v[2] * HAD_SCALE * scale_at(sc.d, 2);
                    o.w = v[3] * HAD_SCALE * scale_at(sc.d, 3);
                    const int q = d->rows[m];
                    float* yr = p.y + (size_t)q * p.D;
                    if (p.ep_world) {   // into the home rank's inbox: slot q of home h is its slot q - h R slots
                        const int per = p.ep_R * p.slots, h = q / per;
                        yr = p.ep_y[h] + (size_t)(q - h * per) * p.D;
                    }
                    *reinterpret_cast<float4*>(yr + n0) = o;
                }
                named_sync(1, CT);
                if (warp == 0) enqueue(1, u, d);
            }
            named_sync(1, CT);   // red and the descriptor are free for the next item
        }
        if (warp == 0) enqueue(2, 0, nullptr);
    }
    // the last CTA to leave resets the entries' readiness (every producer of every CTA is past its waits by then)
    named_sync(3, GWARPS * 32 + 32);
    if (threadIdx.x == 0 && arrive_acq_rel(p.exits) == (int)gridDim.x - 1) {
        for (int i = 0; i < p.maxu; ++i) p.ready[i] = 0;
        *p.exits = 0;
        // every CTA's y stores are ordered before its arrival (release after the CTA barrier above), which this
        // acquire saw: the system-scope release of each home's flag publishes them all
        if (p.ep_world) {
            const int v = *p.ep_epoch + 1;
            for (int h = 0; h < p.ep_world; ++h)
                asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p.ep_flag[h] + p.ep_rank), "r"(v) : "memory");
        }
    }
}

// ------------------------------------------------------------------------------------------------------------------
// The reference's separate epilogue / combine kernels (experts.cu:120-241, 340-393), for drop-in callers of ext().
// ------------------------------------------------------------------------------------------------------------------
__global__ void gateup_epilogue_kernel(const float* __restrict__ Z, const int* __restrict__ pick,
                                       const __half* __restrict__ svh_g, const __half* __restrict__ svh_u,
                                       const __half* __restrict__ suh_d, __half* __restrict__ xd, int P, int N, int SK,
                                       int E, float limit, int act_mode) {
    pdl_launch_dependents();
    pdl_wait();
    const int p = blockIdx.x, blk = blockIdx.y, lane = threadIdx.x;
    const int e = pick[p];
    if (e < 0 || e >= E) return;
    const int n = blk * 128 + 4 * lane;
    float gv[4], uv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float sg = 0.f, su = 0.f;
        for (int s = 0; s < SK; ++s) {
            sg += Z[((size_t)(0 * SK + s) * P + p) * N + n + j];
            su += Z[((size_t)(1 * SK + s) * P + p) * N + n + j];
        }
        gv[j] = sg;
        uv[j] = su;
    }
    fwht128(gv, lane);
    fwht128(uv, lane);
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float act;
        auto bf16r = [](float t) { return __bfloat162float(__float2bfloat16_rn(t)); };
        if (act_mode == 0) {
            const float gg = fminf(bf16r(gv[j] * HAD_SCALE * __half2float(svh_g[(size_t)e * N + n + j])), limit);
            const float uu =
                fminf(fmaxf(bf16r(uv[j] * HAD_SCALE * __half2float(svh_u[(size_t)e * N + n + j])), -limit), limit);
            act = bf16r(bf16r(gg / (1.f + expf(-gg))) * uu);
        } else {
            const float gg = fminf(gv[j] * HAD_SCALE * __half2float(svh_g[(size_t)e * N + n + j]), limit);
            const float uu = fminf(fmaxf(uv[j] * HAD_SCALE * __half2float(svh_u[(size_t)e * N + n + j]), -limit), limit);
            act = gg / (1.f + expf(-gg)) * uu;
        }
        v[j] = __fmul_rn(act, __half2float(suh_d[(size_t)e * N + n + j]));
    }
    fwht128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) xd[(size_t)p * N + n + j] = __float2half_rn(v[j] * HAD_SCALE);
}

// down epilogue (+ optional combine into out / out_shared): y[p] = H(sum of splits) h svh_d; out[row] = sum of the
// first n_routed slots' w * y (fma chain from 0 in slot order), out_shared = w * y of slot n_routed. Block: 32 * slots.
template <typename TOUT>
__global__ void down_combine_kernel(const float* __restrict__ Z, const int* __restrict__ pick,
                                    const __half* __restrict__ svh_d, float* __restrict__ y,
                                    const float* __restrict__ wts, TOUT* __restrict__ out, TOUT* __restrict__ out_shared,
                                    int P, int D, int SK, int E, int slots, int n_routed, int combine) {
    __shared__ float4 part[32][32];
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, blk = blockIdx.y;
    const int k = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blk * 128 + 4 * lane;
    const int p = r * slots + k;
    const int e = pick[p];
    float o[4];
    if (e >= 0 && e < E) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float s = 0.f;
            for (int q = 0; q < SK; ++q) s += Z[((size_t)q * P + p) * D + n + j];
            v[j] = s;
        }
        fwht128(v, lane);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            o[j] = v[j] * HAD_SCALE * __half2float(svh_d[(size_t)e * D + n + j]);
            y[(size_t)p * D + n + j] = o[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = y[(size_t)p * D + n + j];
    }
    if (!combine) return;
    part[k][lane] = make_float4(o[0], o[1], o[2], o[3]);
    __syncthreads();
    if (k == 0) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < n_routed; ++q) {
            const float w = wts[r * slots + q];
            const float4 u = part[q][lane];
            acc[0] = fmaf(w, u.x, acc[0]);
            acc[1] = fmaf(w, u.y, acc[1]);
            acc[2] = fmaf(w, u.z, acc[2]);
            acc[3] = fmaf(w, u.w, acc[3]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) out[(size_t)r * D + n + j] = from_f<TOUT>(acc[j]);
    } else if (k == n_routed && out_shared != nullptr) {
        const float w = wts[r * slots + k];
        const float4 u = part[k][lane];
        out_shared[(size_t)r * D + n + 0] = from_f<TOUT>(w * u.x);
        out_shared[(size_t)r * D + n + 1] = from_f<TOUT>(w * u.y);
        out_shared[(size_t)r * D + n + 2] = from_f<TOUT>(w * u.z);
        out_shared[(size_t)r * D + n + 3] = from_f<TOUT>(w * u.w);
    }
}

// combine (experts.cu:187-195): out[r][d] = sum over slots of fma(w, y) in slot order, fp32.
__global__ void combine_kernel(const float* __restrict__ y, const float* __restrict__ wts, float* __restrict__ out,
                               int D, int slots) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x;
    const int d = blockIdx.y * blockDim.x + threadIdx.x;
    if (d >= D) return;
    float acc = 0.f;
    for (int k = 0; k < slots; ++k) acc = fmaf(wts[r * slots + k], y[((size_t)r * slots + k) * D + d], acc);
    out[(size_t)r * D + d] = acc;
}

// ------------------------------------------------------------------------------------------------------------------
// Expert-parallel combine on a token's home rank: out[r] = sum over the routed slots j < n_routed (slot order, fp32
// fma from 0) of w * y, where y is the slot's row returned by the rank owning its expert (rank of expert e =
// ((e + 1) world - 1) / E_routed, i.e. experts [rank E / world, (rank + 1) E / world)); out_shared[r] = w * y of the
// shared slot (computed on the home rank). The same arithmetic as the single-GPU fused down combine, so the outputs
// are bit-identical for every world size. recv_y: fp32 [world][R][slots][D]. Block (row, 128-column block), a warp.
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(32) ep_combine_kernel(const float* __restrict__ recv_y, const int* __restrict__ pick,
                                                        const float* __restrict__ wts, void* out, void* out_shared,
                                                        int out_dtype, int R, int D, int slots, int n_routed,
                                                        int E_routed, int world, int rank) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, lane = threadIdx.x;
    const int n0 = blockIdx.y * 128 + 4 * lane;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < n_routed; j0 += 8) {   // eight slots' loads in flight, then added in slot order
        float4 y[8];
        bool on[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int j = j0 + q;
            const int e = j < n_routed ? pick[r * slots + j] : -1;
            on[q] = e >= 0 && e < E_routed;
            if (on[q]) {
                const int owner = ((e + 1) * world - 1) / E_routed;
                y[q] = *reinterpret_cast<const float4*>(recv_y + (((size_t)owner * R + r) * slots + j) * D + n0);
            }
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
            if (on[q]) {
                const float w = wts[r * slots + j0 + q];
                acc[0] = fmaf(w, y[q].x, acc[0]);
                acc[1] = fmaf(w, y[q].y, acc[1]);
                acc[2] = fmaf(w, y[q].z, acc[2]);
                acc[3] = fmaf(w, y[q].w, acc[3]);
            }
    }
    store4(out, out_dtype, (size_t)r * D + n0, acc);
    if (out_shared && n_routed < slots) {
        const int j = n_routed;
        float sv[4] = {0.f, 0.f, 0.f, 0.f};
        if (pick[r * slots + j] >= 0) {
            const float w = wts[r * slots + j];
            const float4 y = *reinterpret_cast<const float4*>(recv_y + (((size_t)rank * R + r) * slots + j) * D + n0);
            sv[0] = w * y.x; sv[1] = w * y.y; sv[2] = w * y.z; sv[3] = w * y.w;
        }
        store4(out_shared, out_dtype, (size_t)r * D + n0, sv);
    }
}

size_t grouped_smem(int ntg, int kcap) {
    const int st = gstages(ntg, kcap);
    return (size_t)st * stage_words(ntg, kcap) * 4 + (size_t)red_bytes(ntg) + 2 * st * 8;
}

template <int NTG, int KCAP>
int launch_grouped_t(const GroupedParams& p, dim3 grid, void* stream) {
    auto kern = grouped_kernel<NTG, KCAP>;
    const size_t smem = grouped_smem(NTG, KCAP);
    static bool opted = false;
    if (!opted) {
        if (int rc = allow_smem(kern, smem)) return rc;
        opted = true;
    }
    return launch(kern, grid, dim3(GTHREADS), smem, stream, true, p);
}

int launch_grouped(const GroupedParams& p, int ntg, int kmax, int maxu, void* stream) {
    // persistent: one CTA an SM (never more than the most items a window can have)
    const long long most = (long long)maxu * (p.N / 128) * (p.mode == MODE_Z ? p.mats * p.S : p.S);
    const dim3 grid((unsigned)std::min<long long>(device_sms(), most));
    const long long per_cta = (most + grid.x - 1) / grid.x;
    const int pend_item = p.mode == MODE_DOWN ? p.maxm : 1;
    // static (MODE_Z): the round-robin share of a CTA; dynamic: every item must fit in the CTAs' tables
    ESP_REQUIRE(p.work ? most <= (long long)grid.x * (MAX_PEND / pend_item) : per_cta * pend_item <= MAX_PEND,
                ESP_ERR_INVALID, "grouped: %lld items exceed the deferred-arrival tables", most);
#define ESP_G(N_)                                                                                   \
    return kmax <= 4 ? launch_grouped_t<N_, 4>(p, grid, stream) : launch_grouped_t<N_, 8>(p, grid, stream);
    switch (ntg) {
        case 1: ESP_G(1)
        case 2: ESP_G(2)
        case 3: ESP_G(3)
        default: ESP_G(4)
    }
#undef ESP_G
}

template <int NTG, int KCAP>
int launch_layer_t(const LayerParams& p, dim3 grid, void* stream) {
    auto kern = layer_kernel<NTG, KCAP>;
    const size_t smem = grouped_smem(NTG, KCAP);
    static bool opted = false;
    if (!opted) {
        if (int rc = allow_smem(kern, smem)) return rc;
        opted = true;
    }
    return launch(kern, grid, dim3(LTHREADS), smem, stream, true, p);
}

int launch_layer(const LayerParams& p, int ntg, int kmax, void* stream) {
    const dim3 grid((unsigned)device_sms());   // persistent: one CTA an SM, items handed out dynamically
#define ESP_L(N_) \
    return kmax <= 4 ? launch_layer_t<N_, 4>(p, grid, stream) : launch_layer_t<N_, 8>(p, grid, stream);
    switch (ntg) {
        case 1: ESP_L(1)
        case 2: ESP_L(2)
        case 3: ESP_L(3)
        default: ESP_L(4)
    }
#undef ESP_L
}

int check_tables(const int* k2_host, const int* cb_host, int E, int& kmax) {
    kmax = 0;
    for (int e = 0; e < E; ++e) {
        const int k2 = k2_host[e], cb = cb_host[e];
        ESP_REQUIRE(k2 % 2 == 0 && case_supported(cb, k2 / 2), ESP_ERR_UNSUPPORTED,
                    "expert %d: no grouped instance for codebook %d at K2 %d", e, cb, k2);
        kmax = std::max(kmax, k2 / 2);
    }
    return ESP_OK;
}

}  // namespace
}  // namespace esp

using namespace esp;

extern "C" {

int esp_rot_in(const void* x, int x_dtype, long long x_stride, const int* pick, const uint16_t* suh0,
               const uint16_t* suh1, uint16_t* out0, uint16_t* out1, int rows, int K, int slots, int E, void* stream) {
    ESP_REQUIRE(x && pick && suh0 && suh1 && out0 && out1, ESP_ERR_INVALID, "rot_in: null pointer");
    ESP_REQUIRE(K % 128 == 0 && K > 0, ESP_ERR_INVALID, "K must be a multiple of 128");
    ESP_REQUIRE(x_dtype == ESP_DTYPE_BF16 || x_dtype == ESP_DTYPE_F16, ESP_ERR_INVALID, "x: bf16/fp16 CUDA");
    const int P = rows * slots;
    if (P == 0) return ok();
    const dim3 grid((unsigned)((P * (K / 128) * 2 + 3) / 4));
    int rc;
    if (x_dtype == ESP_DTYPE_BF16)
        rc = launch(rot_in_kernel<__nv_bfloat16>, grid, dim3(128), 0, stream, true,
                    static_cast<const __nv_bfloat16*>(x), x_stride, pick, reinterpret_cast<const __half*>(suh0),
                    reinterpret_cast<const __half*>(suh1), reinterpret_cast<__half*>(out0),
                    reinterpret_cast<__half*>(out1), P, K, slots, E);
    else
        rc = launch(rot_in_kernel<__half>, grid, dim3(128), 0, stream, true, static_cast<const __half*>(x), x_stride,
                    pick, reinterpret_cast<const __half*>(suh0), reinterpret_cast<const __half*>(suh1),
                    reinterpret_cast<__half*>(out0), reinterpret_cast<__half*>(out1), P, K, slots, E);
    if (rc) return rc;
    return ok();
}

// The reference's grouped GEMV: Z[mat][split][p][n] fp32 partial sums (experts.cpp:44-66). k2/cb tables are also
// passed as host copies (k2_host / cb_host, [mats][E]) so the instance set is checked on the host, not trapped on.
int esp_grouped(const uint16_t* X0, const uint16_t* X1, const int64_t* TP0, const int64_t* TP1, const int* B0,
                const int* B1, const int* C0, const int* C1, const int* k2_host, const int* cb_host, int E,
                const int* uids, const int* ucount, const int* members, int maxu, int maxm, float* Z, int mats, int K,
                int N, int P, int SK, int slots, void* stream) {
    ESP_REQUIRE(X0 && TP0 && B0 && C0 && uids && ucount && members && Z && k2_host && cb_host, ESP_ERR_INVALID,
                "grouped: null pointer");
    ESP_REQUIRE(mats == 1 || (mats == 2 && X1 && TP1 && B1 && C1), ESP_ERR_INVALID, "grouped: 1 or 2 matrices");
    ESP_REQUIRE(K % 128 == 0 && N % 128 == 0 && SK >= 1 && (K / 16) >= SK, ESP_ERR_INVALID, "K and N must split evenly");
    ESP_REQUIRE(maxm >= 1 && maxm <= 32 && maxu >= 1, ESP_ERR_INVALID, "grouped: at most 32 members an expert");
    int kmax = 0, km2 = 0;
    if (int rc = check_tables(k2_host, cb_host, E, kmax)) return rc;
    if (mats == 2)
        if (int rc = check_tables(k2_host + E, cb_host + E, E, km2)) return rc;
    GroupedParams p = {};
    p.tp[0] = TP0; p.tp[1] = mats == 2 ? TP1 : TP0;
    p.k2[0] = B0; p.k2[1] = mats == 2 ? B1 : B0;
    p.cb[0] = C0; p.cb[1] = mats == 2 ? C1 : C0;
    p.X[0] = reinterpret_cast<const __half*>(X0);
    p.X[1] = reinterpret_cast<const __half*>(mats == 2 ? X1 : X0);
    p.uids = uids; p.ucount = ucount; p.members = members;
    p.maxm = maxm; p.slots = slots; p.K = K; p.N = N; p.P = P; p.S = SK; p.mats = mats; p.mode = MODE_Z; p.E = E;
    p.Z = Z;
    if (int rc = launch_grouped(p, (maxm + 7) / 8, std::max(kmax, km2), maxu, stream)) return rc;
    return ok();
}

// Fused gate + up + SwiGLU epilogue: xd[p] for every slot with a valid expert (experts.py routed2 launches 3-4).
int esp_moe_gateup(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u,
                   const int* k2_g, const int* k2_u, const int* cb_g, const int* cb_u, const int* k2_host,
                   const int* cb_host, int E, const uint16_t* svh_g, const uint16_t* svh_u, const uint16_t* suh_d,
                   const int* uids, const int* ucount, const int* members, int maxu, int maxm, int slots, int P, int D,
                   int I, int S, float* Z, int* counters, uint16_t* xd, void* stream) {
    ESP_REQUIRE(xg && xu && tp_g && tp_u && svh_g && svh_u && suh_d && uids && ucount && members && xd && k2_host &&
                    cb_host,
                ESP_ERR_INVALID, "moe_gateup: null pointer");
    ESP_REQUIRE(D % 128 == 0 && I % 128 == 0 && S >= 1 && D / 16 >= S, ESP_ERR_INVALID, "moe_gateup: shapes");
    ESP_REQUIRE(S == 1 || (Z && counters), ESP_ERR_SCRATCH, "moe_gateup: split partials need Z and counters");
    ESP_REQUIRE(maxm >= 1 && maxm <= 32 && maxu >= 1, ESP_ERR_INVALID, "moe_gateup: at most 32 members an expert");
    int k1 = 0, k2m = 0;
    if (int rc = check_tables(k2_host, cb_host, E, k1)) return rc;
    if (int rc = check_tables(k2_host + E, cb_host + E, E, k2m)) return rc;
    GroupedParams p = {};
    p.tp[0] = tp_g; p.tp[1] = tp_u; p.k2[0] = k2_g; p.k2[1] = k2_u; p.cb[0] = cb_g; p.cb[1] = cb_u;
    p.X[0] = reinterpret_cast<const __half*>(xg);
    p.X[1] = reinterpret_cast<const __half*>(xu);
    p.uids = uids; p.ucount = ucount; p.members = members;
    p.maxm = maxm; p.slots = slots; p.K = D; p.N = I; p.P = P; p.S = S; p.mats = 2; p.mode = MODE_GATEUP; p.E = E;
    p.Z = Z; p.counters = counters;
    p.work = counters ? counters + (size_t)maxu * (I / 128) : nullptr;   // the item counter after the arrivals
    p.svh_g = reinterpret_cast<const __half*>(svh_g);
    p.svh_u = reinterpret_cast<const __half*>(svh_u);
    p.suh_d = reinterpret_cast<const __half*>(suh_d);
    p.xd = reinterpret_cast<__half*>(xd);
    if (int rc = launch_grouped(p, (maxm + 7) / 8, std::max(k1, k2m), maxu, stream)) return rc;
    return ok();
}

// Fused down + combine: out[row] (routed sum, slot order) and out_shared[row] (gated shared slot) in out_dtype.
int esp_moe_down(const uint16_t* xd, const int64_t* tp_d, const int* k2_d, const int* cb_d, const int* k2_host,
                 const int* cb_host, int E, const uint16_t* svh_d, const int* uids, const int* ucount,
                 const int* members, int maxu, int maxm, const int* pick, const float* wts, int slots, int n_routed,
                 int rows, int I, int D, float* y, int* counters, void* out, void* out_shared, int out_dtype,
                 void* stream) {
    ESP_REQUIRE(xd && tp_d && svh_d && uids && ucount && members && pick && wts && y && counters && out && k2_host &&
                    cb_host,
                ESP_ERR_INVALID, "moe_down: null pointer");
    ESP_REQUIRE(D % 128 == 0 && I % 128 == 0, ESP_ERR_INVALID, "moe_down: shapes");
    ESP_REQUIRE(maxm >= 1 && maxm <= 32 && maxu >= 1 && slots >= 1 && slots <= 32 && n_routed <= slots &&
                    D / 128 <= 256,
                ESP_ERR_INVALID, "moe_down: limits (32 members, 32 slots, D <= 32768)");
    ESP_REQUIRE(out_dtype >= 0 && out_dtype <= 2, ESP_ERR_INVALID, "moe_down: dtype");
    int kmax = 0;
    if (int rc = check_tables(k2_host, cb_host, E, kmax)) return rc;
    GroupedParams p = {};
    p.tp[0] = p.tp[1] = tp_d; p.k2[0] = p.k2[1] = k2_d; p.cb[0] = p.cb[1] = cb_d;
    p.X[0] = p.X[1] = reinterpret_cast<const __half*>(xd);
    p.uids = uids; p.ucount = ucount; p.members = members;
    p.maxm = maxm; p.slots = slots; p.K = I; p.N = D; p.P = rows * slots; p.S = 1; p.mats = 1; p.mode = MODE_DOWN;
    p.E = E; p.counters = counters;
    p.work = counters + (size_t)rows * (D / 128);                          // the item counter after the arrivals
    p.svh_d = reinterpret_cast<const __half*>(svh_d);
    p.pick = pick; p.wts = wts; p.y = y; p.out = out; p.out_shared = out_shared; p.out_dtype = out_dtype;
    p.n_routed = n_routed;
    if (int rc = launch_grouped(p, (maxm + 7) / 8, kmax, maxu, stream)) return rc;
    return ok();
}

// The fused expert layer in one launch: gate/up + SwiGLU and down + combine (the sequence of esp_moe_gateup and
// esp_moe_down, the same output bits).
static int moe_layer_impl(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u, const int64_t* tp_d,
                  const int* k2_g, const int* k2_u, const int* k2_d, const int* cb_g, const int* cb_u, const int* cb_d,
                  const int* k2_host, const int* cb_host, int E, const uint16_t* svh_g, const uint16_t* svh_u,
                  const uint16_t* suh_d, const uint16_t* svh_d, const int* uids, const int* ucount, const int* members,
                  int maxu, int maxm, const int* pick, const float* wts, int slots, int n_routed, int rows, int D, int I,
                  int S, float* Z, uint16_t* xd, float* y, int* counters, void* out, void* out_shared, int out_dtype,
                  void* stream, const LayerParams* ep) {
    ESP_REQUIRE(xg && xu && tp_g && tp_u && tp_d && k2_g && k2_u && k2_d && cb_g && cb_u && cb_d && k2_host &&
                    cb_host && svh_g && svh_u && suh_d && svh_d && uids && ucount && members && pick && wts && xd &&
                    y && counters && out,
                ESP_ERR_INVALID, "moe_layer: null pointer");
    ESP_REQUIRE(D % 128 == 0 && I % 128 == 0 && S >= 1 && D / 16 >= S && D / 128 <= 256, ESP_ERR_INVALID,
                "moe_layer: shapes");
    ESP_REQUIRE(S == 1 || Z, ESP_ERR_SCRATCH, "moe_layer: split partials need Z");
    ESP_REQUIRE(maxm >= 1 && maxm <= 32 && maxu >= 1 && slots >= 1 && slots <= 32 && n_routed <= slots && rows >= 0 &&
                    rows <= 32,
                ESP_ERR_INVALID, "moe_layer: limits (32 rows, 32 members, 32 slots)");
    ESP_REQUIRE(out_dtype >= 0 && out_dtype <= 2, ESP_ERR_INVALID, "moe_layer: dtype");
    int km = 0, kmax = 0;
    for (int t = 0; t < 3; ++t) {
        if (int rc = check_tables(k2_host + t * E, cb_host + t * E, E, km)) return rc;
        kmax = std::max(kmax, km);
    }
    LayerParams p = {};
    p.uids = uids; p.ucount = ucount; p.members = members;
    p.maxm = maxm; p.maxu = maxu; p.slots = slots; p.rows = rows; p.E = E; p.n_routed = n_routed;
    p.tp[0] = tp_g; p.tp[1] = tp_u; p.tp[2] = tp_d;
    p.k2[0] = k2_g; p.k2[1] = k2_u; p.k2[2] = k2_d;
    p.cb[0] = cb_g; p.cb[1] = cb_u; p.cb[2] = cb_d;
    p.xg = reinterpret_cast<const __half*>(xg);
    p.xu = reinterpret_cast<const __half*>(xu);
    p.D = D; p.I = I; p.S = S;
    p.svh_g = reinterpret_cast<const __half*>(svh_g);
    p.svh_u = reinterpret_cast<const __half*>(svh_u);
    p.suh_d = reinterpret_cast<const __half*>(suh_d);
    p.Z = Z;
    p.xd = reinterpret_cast<__half*>(xd);
    p.svh_d = reinterpret_cast<const __half*>(svh_d);
    p.pick = pick; p.wts = wts; p.y = y; p.out = out; p.out_shared = out_shared; p.out_dtype = out_dtype;
    p.cnt_gu = counters;
    p.cnt_d = p.cnt_gu + (size_t)maxu * (I / 128);
    p.work = p.cnt_d + (size_t)rows * (D / 128);
    p.ready = p.work + 1;
    p.exits = p.ready + maxu;
    if (ep) {
        for (int h = 0; h < 8; ++h) {
            p.ep_y[h] = ep->ep_y[h];
            p.ep_flag[h] = ep->ep_flag[h];
        }
        p.ep_epoch = ep->ep_epoch;
        p.ep_world = ep->ep_world;
        p.ep_rank = ep->ep_rank;
        p.ep_R = ep->ep_R;
    }
    if (int rc = launch_layer(p, (maxm + 7) / 8, kmax, stream)) return rc;
    return ok();
}

int esp_moe_layer(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u, const int64_t* tp_d,
                  const int* k2_g, const int* k2_u, const int* k2_d, const int* cb_g, const int* cb_u, const int* cb_d,
                  const int* k2_host, const int* cb_host, int E, const uint16_t* svh_g, const uint16_t* svh_u,
                  const uint16_t* suh_d, const uint16_t* svh_d, const int* uids, const int* ucount, const int* members,
                  int maxu, int maxm, const int* pick, const float* wts, int slots, int n_routed, int rows, int D, int I,
                  int S, float* Z, uint16_t* xd, float* y, int* counters, void* out, void* out_shared, int out_dtype,
                  void* stream) {
    return moe_layer_impl(xg, xu, tp_g, tp_u, tp_d, k2_g, k2_u, k2_d, cb_g, cb_u, cb_d, k2_host, cb_host, E, svh_g, svh_u,
                          suh_d, svh_d, uids, ucount, members, maxu, maxm, pick, wts, slots, n_routed, rows, D, I, S, Z,
                          xd, y, counters, out, out_shared, out_dtype, stream, nullptr);
}

int esp_moe_layer_ep(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u,
                     const int64_t* tp_d, const int* k2_g, const int* k2_u, const int* k2_d, const int* cb_g,
                     const int* cb_u, const int* cb_d, const int* k2_host, const int* cb_host, int E,
                     const uint16_t* svh_g, const uint16_t* svh_u, const uint16_t* suh_d, const uint16_t* svh_d,
                     const int* uids, const int* ucount, const int* members, int maxu, int maxm,
                     const int* local_pick, const float* no_w, int slots, int rows, int D, int I, int S, float* Z,
                     uint16_t* xd, int* counters, float* const* inbox_y, int* const* flags_y, const int* epoch,
                     int world, int rank, int R, float* scratch_out, void* stream) {
    ESP_REQUIRE(inbox_y && flags_y && epoch && scratch_out && local_pick && no_w, ESP_ERR_INVALID,
                "moe_layer_ep: null pointer");
    ESP_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world && R >= 1 && rows == world * R, ESP_ERR_INVALID,
                "moe_layer_ep: rows = world * R, 1 to 8 ranks");
    LayerParams ep = {};
    for (int h = 0; h < world; ++h) {
        ESP_REQUIRE(inbox_y[h] && flags_y[h], ESP_ERR_INVALID, "moe_layer_ep: rank %d's inbox", h);
        ep.ep_y[h] = inbox_y[h];
        ep.ep_flag[h] = flags_y[h];
    }
    ep.ep_epoch = epoch;
    ep.ep_world = world;
    ep.ep_rank = rank;
    ep.ep_R = R;
    // no combine on this rank (n_routed 0): the finisher still counts each row's slots (the local picks) and leaves
    // its counters zero; its row outputs go to scratch_out ([rows][D] fp32, unread)
    return moe_layer_impl(xg, xu, tp_g, tp_u, tp_d, k2_g, k2_u, k2_d, cb_g, cb_u, cb_d, k2_host, cb_host, E, svh_g, svh_u,
                          suh_d, svh_d, uids, ucount, members, maxu, maxm, local_pick, no_w, slots, 0, rows, D, I, S, Z,
                          xd, scratch_out, counters, scratch_out, nullptr, ESP_DTYPE_F32, stream, &ep);
}

size_t esp_moe_layer_counters(int maxu, int rows, int D, int I) {
    return (size_t)maxu * (I / 128) + (size_t)rows * (D / 128) + 2 + (size_t)maxu;
}

int esp_gateup_epilogue(const float* Z, const int* pick, const uint16_t* svh_g, const uint16_t* svh_u,
                        const uint16_t* suh_d, uint16_t* xd, int rows, int P, int N, int SK, int slots, int E,
                        float limit, int act_mode, void* stream) {
    ESP_REQUIRE(Z && pick && svh_g && svh_u && suh_d && xd, ESP_ERR_INVALID, "gateup_epilogue: null pointer");
    ESP_REQUIRE(N % 128 == 0, ESP_ERR_INVALID, "N must be a multiple of 128");
    if (rows * slots == 0) return ok();
    if (int rc = launch(gateup_epilogue_kernel, dim3((unsigned)(rows * slots), (unsigned)(N / 128)), dim3(32), 0,
                        stream, true, Z, pick, reinterpret_cast<const __half*>(svh_g),
                        reinterpret_cast<const __half*>(svh_u), reinterpret_cast<const __half*>(suh_d),
                        reinterpret_cast<__half*>(xd), P, N, SK, E, limit, act_mode))
        return rc;
    return ok();
}

// down_epilogue (combine = 0, out unused), down_combine (fp32 out), down_combine2 (out in out_dtype + out_shared)
int esp_down_combine(const float* Z, const int* pick, const uint16_t* svh_d, float* y, const float* wts, void* out,
                     void* out_shared, int out_dtype, int rows, int P, int D, int SK, int slots, int E, int n_routed,
                     int combine, void* stream) {
    ESP_REQUIRE(Z && pick && svh_d && y, ESP_ERR_INVALID, "down_combine: null pointer");
    ESP_REQUIRE(!combine || (wts && out), ESP_ERR_INVALID, "down_combine: weights and out needed");
    ESP_REQUIRE(slots >= 1 && slots <= 32 && n_routed <= slots, ESP_ERR_INVALID, "at most 32 slots a row");
    ESP_REQUIRE(D % 128 == 0, ESP_ERR_INVALID, "D must be a multiple of 128");
    if (rows == 0) return ok();
    const dim3 grid((unsigned)rows, (unsigned)(D / 128)), block((unsigned)(32 * slots));
    const __half* sv = reinterpret_cast<const __half*>(svh_d);
    int rc;
    if (out_dtype == ESP_DTYPE_BF16)
        rc = launch(down_combine_kernel<__nv_bfloat16>, grid, block, 0, stream, true, Z, pick, sv, y, wts,
                    static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(out_shared), P, D, SK, E, slots,
                    n_routed, combine);
    else if (out_dtype == ESP_DTYPE_F16)
        rc = launch(down_combine_kernel<__half>, grid, block, 0, stream, true, Z, pick, sv, y, wts,
                    static_cast<__half*>(out), static_cast<__half*>(out_shared), P, D, SK, E, slots, n_routed, combine);
    else
        rc = launch(down_combine_kernel<float>, grid, block, 0, stream, true, Z, pick, sv, y, wts,
                    static_cast<float*>(out), static_cast<float*>(out_shared), P, D, SK, E, slots, n_routed, combine);
    if (rc) return rc;
    return ok();
}

int esp_ep_combine(const float* recv_y, const int* pick, const float* wts, void* out, void* out_shared, int out_dtype,
                   int R, int D, int slots, int n_routed, int E_routed, int world, int rank, void* stream) {
    ESP_REQUIRE(recv_y && pick && wts && out, ESP_ERR_INVALID, "ep_combine: null pointer");
    ESP_REQUIRE(D % 128 == 0 && slots >= 1 && slots <= 32 && n_routed <= slots && E_routed >= 1 && world >= 1 &&
                    rank >= 0 && rank < world && out_dtype >= 0 && out_dtype <= 2,
                ESP_ERR_INVALID, "ep_combine: limits");
    if (R == 0) return ok();
    if (int rc = launch(ep_combine_kernel, dim3((unsigned)R, (unsigned)(D / 128)), dim3(32), 0, stream, true, recv_y, pick,
                        wts, out, out_shared, out_dtype, R, D, slots, n_routed, E_routed, world, rank))
        return rc;
    return ok();
}

int esp_wait_flag(const int* flag, int need, int* result, void* stream) {
    ESP_REQUIRE(flag && result, ESP_ERR_INVALID, "wait_flag: null pointer");
    if (int rc = launch(wait_flag_kernel, dim3(1), dim3(32), 0, stream, false, flag, need, result)) return rc;
    return ok();
}

int esp_combine(const float* y, const float* wts, float* out, int rows, int D, int slots, void* stream) {
    ESP_REQUIRE(y && wts && out, ESP_ERR_INVALID, "combine: null pointer");
    if (rows == 0) return ok();
    if (int rc = launch(combine_kernel, dim3((unsigned)rows, (unsigned)((D + 255) / 256)), dim3(256), 0, stream, true,
                        y, wts, out, D, slots))
        return rc;
    return ok();
}

}  // extern "C"
