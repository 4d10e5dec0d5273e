// Dense layer decode for 1..32 rows: every matrix of one layer (q/k/v, in_proj_qkv/z, o, the head) in one
// persistent launch that streams the compressed trellis once and decodes each weight once for all rows.
//
// Reference behaviour (vllm_espalier/csrc/dense.cu:130-238, ops.py, dense.py): y_s = H(H(x * suh_s) @ W_s) * svh_s
// written into columns col0_s of y, fp16 rotated activations, fp32 sums, output in the model's dtype; rows are
// independent, split and warp ranges depend on the shape alone, every sum runs in a fixed order.
//
// B200 design:
//   * rot_kernel writes fp16 H(x * suh_s) / sqrt(128) for every matrix once, in a tile-major layout
//     [s][k-tile][k-half][row][8] whose per-k-tile slice is one contiguous run of 16-byte copies (and bank-conflict free as an MMA
//     B fragment).
//   * dense_kernel: one CTA per SM. The layer is a list of units (128-column block, 16-row k-tile) in block-major
//     order, split into G contiguous ranges, one per CTA: with fewer blocks than SMs, S = SMs / blocks equal k-slices
//     of every block (G = blocks * S, one segment a CTA); otherwise G = SMs equal ranges over whole blocks. Two
//     producer warps (the even and the odd units of each stage; one warp sharing a scheduler with four busy consumer
//     warps could not keep the ring filled) stream each unit's 8 tiles (8K words each) and its activation slice into a
//     ring of shared-memory stages with 16-byte cp.async from all 32 lanes, completing on mbarriers (a bulk copy a
//     unit measured ~40 ns of TMA issue each, too slow for 1 KB units). 16 consumer warps in two groups (alternate
//     units) decode tile w of every unit straight into the A fragment of mma.sync m16n8k16 (M = 16 output columns,
//     N = 8 tokens), i.e. each weight is decoded once whatever the number of rows.
//   * A block whose k range spans several CTAs' ranges is finished by the CTA holding its first k-tile (for which it is
//     the last segment); every other CTA of the block holds it as its first segment and stores that partial, as
//     tagged 64-bit words (value | 1 << 32), in its one slot of Z. The finisher reads the slots in CTA (= k) order,
//     polling each word's tag (bounded), adds them after its own sums, and clears the slots to zero for the next
//     launch: no fence, no atomic, and the other CTAs leave as soon as their stores are issued. With equal k-slices
//     (S CTAs a block, the default below SMs blocks) and more than 8 rows the S CTAs share the finishing instead:
//     slice j stores the rows it does not finish and finishes the rows r = j (mod S). The sums are the same either
//     way (k order from 0). A block inside one CTA's range is finished in place. Finishing = FWHT-128 of the sums, * step, * H/sqrt(128) * svh, in the
//     reference's order, then the store in y's dtype. The ranges depend on the shape and the SM count only.
//   * Decode ahead (fused path): the weights do not depend on the previous kernel, so a CTA decodes its units into
//     shared memory before the launch wait while the previous launch drains; when every unit of every CTA fits, all
//     of them are (the wait is then followed by the rotations, the products and the finishing alone).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host.hpp"
#include "trellis.cuh"

ESP_DEFINE_STATUS_READER(dense)

namespace esp {
namespace {

constexpr int MAX_SHARDS = 4;
#ifndef ESP_DENSE_GROUPS
#define ESP_DENSE_GROUPS 2
#endif
constexpr int GROUPS = ESP_DENSE_GROUPS;       // consumer groups of 8 warps, taking alternate units of a stage
constexpr int CWARPS = 8 * GROUPS;             // consumer warps: warp w decodes tile w % 8 of its group's units
#ifndef ESP_DENSE_PRODUCERS
#define ESP_DENSE_PRODUCERS 2
#endif
constexpr int PRODUCERS = ESP_DENSE_PRODUCERS;  // producer warps: unit j of a stage goes to producer j % PRODUCERS
constexpr int THREADS = (CWARPS + PRODUCERS) * 32;
#ifndef ESP_DENSE_BULK
#define ESP_DENSE_BULK 0
#endif
// 1: the fused path's producers move each unit with one 1-D bulk copy (cp.async.bulk, mbarrier transaction count)
// from one lane instead of 16-byte cp.async from all lanes (a measured alternative; off by default)
constexpr bool BULK = ESP_DENSE_BULK != 0;
constexpr int UPS = 8;                         // units per pipeline stage
constexpr int STAGES = 6;                      // pipeline depth (stages of UPS units)
constexpr int RED_STRIDE = 132;                // fp32 row stride of the reduction buffer (bank-conflict free)
#ifndef ESP_DENSE_CTAS_PER_SM
#define ESP_DENSE_CTAS_PER_SM 1
#endif
constexpr int CTAS_PER_SM = ESP_DENSE_CTAS_PER_SM;   // CTAs a launch puts on a streaming multiprocessor
#ifndef ESP_DENSE_RESIDENT
#define ESP_DENSE_RESIDENT ESP_DENSE_CTAS_PER_SM
#endif
// CTAs the resources of one are sized for on a streaming multiprocessor (registers, shared memory): more than
// CTAS_PER_SM lets the next launch's CTAs become resident beside this one's and decode ahead while it runs
constexpr int RESIDENT = ESP_DENSE_RESIDENT;
static_assert(RESIDENT >= CTAS_PER_SM, "a launch's CTAs must fit");

struct DShard {
    const uint32_t* T;   // trellis words [K/16][N/16][8K]
    const __half* suh;   // [K]
    const __half* svh;   // [N]
    int nb0;             // first 128-column block of this matrix among all blocks of the launch
    int nb;              // its blocks
    int col0;            // its first output column in y
};

struct DenseParams {
    DShard s[MAX_SHARDS];
    int n;                       // matrices
    const __half* xh;            // rotated activations [n][KT][2][Mp][8] (rot_kernel path)
    const void* x;               // the layer input (fused-rotation path)
    int x_dtype;
    long long x_stride;
    int xh_chunks;               // fused path: 128-input chunks the shared rotation buffer holds
    void* y;
    int y_dtype;
    long long y_stride;
    uint64_t* Z;                 // tagged partial sums [G][M][128]: CTA c's first segment; zero on entry and exit
    int* counters;               // [blocks], zero (the reference's argument; not written by this kernel)
    int M, Mp, K, KT, U, G;      // rows, padded rows, inputs, k tiles, units, CTAs (G <= U)
    int NB;                      // 128-column blocks
    int S;                       // > 1: the S CTAs of a block form a thread-block cluster (block-aligned k-slices)
    float scale;                 // codebook step of the kernel form
    int npre;                    // fused path: units decoded ahead of the launch wait (whole stages, one segment)
    int ahead_all;               // fused path: every CTA decodes all of its units ahead of the wait (npre = max)
    int kslices;                 // > 1: G = blocks * kslices equal k-slices (CTA c = block c / S, slice c % S)
    int stages;                  // ring depth in stages (<= STAGES)
};

struct RotParams {
    const void* x;
    int x_dtype;
    long long x_stride;
    const __half* suh[MAX_SHARDS];
    __half* xh;
    int M, Mp, K, KT;
};

// ------------------------------------------------------------------------------------------------------------------
// xh[s][kt][h][m][e] = fp16(FWHT(x[m] * suh_s) * H) for k = 16 kt + 8 h + e (zero rows for m >= M): dense.cu:92-117
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) rot_kernel(const __grid_constant__ RotParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 4 + warp, m = blockIdx.y, s = blockIdx.z;
    if (blk * 128 >= p.K) return;
    const int k = blk * 128 + 4 * lane;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (m < p.M) {
        load4(p.x, p.x_dtype, (size_t)m * p.x_stride + k, v);
        const uint2 su = *reinterpret_cast<const uint2*>(p.suh[s] + k);
        const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&su.x));
        const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&su.y));
        v[0] = __fmul_rn(v[0], s01.x); v[1] = __fmul_rn(v[1], s01.y);
        v[2] = __fmul_rn(v[2], s23.x); v[3] = __fmul_rn(v[3], s23.y);
    }
    fwht128(v, lane);
    const __half2 a = __floats2half2_rn(v[0] * HAD_SCALE, v[1] * HAD_SCALE);
    const __half2 b = __floats2half2_rn(v[2] * HAD_SCALE, v[3] * HAD_SCALE);
    const int kt = k >> 4, h = (k >> 3) & 1, e = k & 7;
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p.xh + ((((size_t)s * p.KT + kt) * 2 + h) * p.Mp + m) * 8 + e) = u;
}

// First unit of CTA c: the units (block-major, k-tile minor) split in G equal contiguous ranges (with G = blocks * S
// these are the S k-slices of every block). U * G < 2^31 is checked on the host, so 32-bit arithmetic is exact.
__device__ __forceinline__ int range_start(int c, const DenseParams& p) { return c * p.U / p.G; }
// The CTA whose range holds unit u (the largest c with range_start(c) <= u).
__device__ __forceinline__ int cta_of(int u, const DenseParams& p) { return ((u + 1) * p.G - 1) / p.U; }

__device__ __forceinline__ uint2 load_svh(const DShard& S, int bl, int lane) {
    return *reinterpret_cast<const uint2*>(S.svh + bl * 128 + 4 * lane);
}

// The finished 4 outputs of lane `lane` of one row of a 128-column block (dense.cu:120-128) and their store.
__device__ __forceinline__ void finish_store(float (&v)[4], int lane, const DShard& S, int bl, int row,
                                             const DenseParams& p, uint2 sv) {
    fwht128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= p.scale;
    const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
    const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
    v[0] *= HAD_SCALE * s01.x; v[1] *= HAD_SCALE * s01.y; v[2] *= HAD_SCALE * s23.x; v[3] *= HAD_SCALE * s23.y;
    store4(p.y, p.y_dtype, (size_t)row * p.y_stride + S.col0 + bl * 128 + 4 * lane, v);
}

__device__ __forceinline__ int shard_of(int bg, const DenseParams& p) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < MAX_SHARDS; ++i)
        if (i < p.n && bg >= p.s[i].nb0) s = i;
    return s;
}

// Tagged partial sums: TAG marks a word written by the launch in flight; a consumed slot is cleared to zero.
constexpr uint64_t TAG = 1ull << 32;
// Poll 4 tagged words until all carry the tag; gives up after WAIT_NS (recording ESP_ERR_TIMEOUT, values then 0).
__device__ __forceinline__ float4 poll_tagged4(const uint64_t* w) {
    const uint64_t t0 = global_ns();
    while (true) {
        uint64_t a, b, c, d;
        ld_relaxed_v2_u64(w, a, b);
        ld_relaxed_v2_u64(w + 2, c, d);
        if (((a & b & c & d) >> 32) != 0)
            return make_float4(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b), __uint_as_float((uint32_t)c),
                               __uint_as_float((uint32_t)d));
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS || (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT)) {
            report(ESP_ERR_TIMEOUT);
            return make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// Row r of a block split over the n CTAs c0..c0 + n - 1 (k order), finished by CTA c0 + own: the n partials added in
// k order from 0 (this CTA's own from red, the others' tagged Z slots, four reads in flight, a word whose tag is not
// set yet polled, bounded), each slot row read cleared for the next launch; then the block's finishing and store.
__device__ __forceinline__ void finish_row(const DenseParams& p, const float* red, int c0, int n, int own, int r,
                                           const DShard& S, int bl, uint2 sv, int lane) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int q4 = 0; q4 < n; q4 += 4) {
        float4 f[4];
        uint32_t ok = 0;
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int q = q4 + d;
            if (q < n && q != own) {
                const uint64_t* w = p.Z + ((size_t)(c0 + q) * p.M + r) * 128 + 4 * lane;
                uint64_t a, b, cc, dd;
                ld_relaxed_v2_u64(w, a, b);
                ld_relaxed_v2_u64(w + 2, cc, dd);
                f[d] = make_float4(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b),
                                   __uint_as_float((uint32_t)cc), __uint_as_float((uint32_t)dd));
                ok |= (((a & b & cc & dd) >> 32) != 0 ? 1u : 0u) << d;
            }
        }
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int q = q4 + d;
            if (q >= n) break;
            if (q == own) {
                f[d] = *reinterpret_cast<const float4*>(red + r * RED_STRIDE + 4 * lane);
            } else {
                uint64_t* w = p.Z + ((size_t)(c0 + q) * p.M + r) * 128 + 4 * lane;
                if (!((ok >> d) & 1u)) f[d] = poll_tagged4(w);
                st_relaxed_v2_u64(w, 0ull, 0ull);       // the slot row is empty again
                st_relaxed_v2_u64(w + 2, 0ull, 0ull);
            }
            v[0] += f[d].x; v[1] += f[d].y; v[2] += f[d].z; v[3] += f[d].w;
        }
    }
    finish_store(v, lane, S, bl, r, p, sv);
}

// This CTA's partial rows (red) in its Z slot as tagged words, the rows r with skip(r) false.
template <typename Skip>
__device__ __forceinline__ void store_partial(const DenseParams& p, const float* red, int c, int warp, int lane,
                                              Skip skip) {
    uint64_t* zs = p.Z + (size_t)c * p.M * 128;
    for (int r = warp; r < p.M; r += CWARPS) {
        if (skip(r)) continue;
        const float4 q = *reinterpret_cast<const float4*>(red + r * RED_STRIDE + 4 * lane);
        uint64_t* w = zs + r * 128 + 4 * lane;
        st_relaxed_v2_u64(w, TAG | __float_as_uint(q.x), TAG | __float_as_uint(q.y));
        st_relaxed_v2_u64(w + 2, TAG | __float_as_uint(q.z), TAG | __float_as_uint(q.w));
    }
}

// fp16 H(x[row] * suh) / sqrt(128) of 128-input chunks, stored as MMA B-fragment slices (k-tile, k-half, row, 8): the
// rot_kernel arithmetic (bit-identical), by one warp into shared memory. Items it = row + MP * chunk_offset; the warp's
// items are loaded in batches of RB before their transforms so the global-load latency is paid once a batch.
template <int MP>
__device__ __forceinline__ void rotate_items(const DenseParams& p, const __half* suh, int chunk0, int nch, int warp,
                                             int lane, __half* xrot) {
    constexpr int RB = 4;
    const int ktl = lane >> 2, h = (lane >> 1) & 1, e = (lane & 1) * 4;     // k = chunk*128 + 16 ktl + 8 h + e
    const int items = nch * p.M;                                            // real rows only (rows >= M stay zero)
    for (int base = warp; base < items; base += RB * CWARPS) {
        float v[RB][4];
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            const int it = base + r * CWARPS, row = it % p.M, ch = chunk0 + it / p.M;
            v[r][0] = v[r][1] = v[r][2] = v[r][3] = 0.f;
            if (it < items) {
                const int k = ch * 128 + 4 * lane;
                load4(p.x, p.x_dtype, (size_t)row * p.x_stride + k, v[r]);
                const uint2 su = *reinterpret_cast<const uint2*>(suh + k);
                const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&su.x));
                const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&su.y));
                v[r][0] = __fmul_rn(v[r][0], s01.x); v[r][1] = __fmul_rn(v[r][1], s01.y);
                v[r][2] = __fmul_rn(v[r][2], s23.x); v[r][3] = __fmul_rn(v[r][3], s23.y);
            }
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            const int it = base + r * CWARPS, row = it % p.M, cl = it / p.M;
            if (it >= items) break;
            fwht128(v[r], lane);
            const __half2 a = __floats2half2_rn(v[r][0] * HAD_SCALE, v[r][1] * HAD_SCALE);
            const __half2 b = __floats2half2_rn(v[r][2] * HAD_SCALE, v[r][3] * HAD_SCALE);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(xrot + (size_t)cl * 8 * 2 * MP * 8 + ((ktl * 2 + h) * MP + row) * 8 + e) = u;
        }
    }
}

template <int CB, int K, int NTG, bool FUSED>
__global__ void __launch_bounds__(THREADS, RESIDENT) dense_kernel(const __grid_constant__ DenseParams p) {
    constexpr int TW = 8 * K;                          // words a tile
    constexpr int UNIT_W = 8 * TW;                     // words a unit (8 tiles)
    constexpr int MP = 8 * NTG;
    constexpr int SLICE_W = MP * 8;                    // words of a k-tile's activation slice
    constexpr int STAGE_W = UPS * (UNIT_W + (FUSED ? 0 : SLICE_W));
    constexpr bool BULKW = FUSED && BULK;
    extern __shared__ __align__(128) uint32_t smem[];
    float* red = reinterpret_cast<float*>(smem + (size_t)p.stages * STAGE_W);   // [MP][RED_STRIDE]
    uint32_t* xrot = reinterpret_cast<uint32_t*>(red + MP * RED_STRIDE);      // fused: [chunks][8][2][MP][4]
    uint4* pre = reinterpret_cast<uint4*>(xrot + (FUSED ? (size_t)p.xh_chunks * 8 * SLICE_W : 0));  // [npre][8][32]
    uint64_t* full = reinterpret_cast<uint64_t*>(pre + (FUSED ? (size_t)p.npre * 8 * 32 : 0));
    uint64_t* empty = full + STAGES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const int u0 = range_start(c, p), u1 = range_start(c + 1, p);
    const int n = u1 - u0;
    const int nst = (n + UPS - 1) / UPS;
    const int bg0 = u0 / p.KT, kt0 = u0 - bg0 * p.KT;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            // one arrival a producer lane when its copies have landed; bulk copies: one a producer, with its bytes
            mbar_init(&full[i], BULKW ? PRODUCERS : 32 * PRODUCERS);
            mbar_init(&empty[i], CWARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp >= CWARPS) {   // -------- producer warps: 16-byte async copies, all lanes, arrival on the stage's barrier --------
        // producer pw copies units j = pw, pw + PRODUCERS, ... of each stage (the CTA's units u0 + pw + PRODUCERS i):
        // their UNIT_W words in 16-byte pieces spread over the 32 lanes (and their activation slices)
        const int pw = warp - CWARPS;
        const uint32_t sbase = smem_addr(smem);
        struct Cur { int bg, kt, s; };
        auto start = [&]() -> Cur {
            Cur q{bg0, kt0 + pw, shard_of(bg0, p)};
            if (q.kt >= p.KT) {
                q.kt -= p.KT;
                ++q.bg;
                if (q.s + 1 < p.n && q.bg >= p.s[q.s + 1].nb0) ++q.s;
            }
            return q;
        };
        auto step2 = [&](Cur& q) {   // PRODUCERS units on
            q.kt += PRODUCERS;
            if (q.kt >= p.KT) {
                q.kt -= p.KT;
                ++q.bg;
                if (q.s + 1 < p.n && q.bg >= p.s[q.s + 1].nb0) ++q.s;
            }
        };
        auto src_w = [&](const Cur& q) -> const uint32_t* {
            const DShard& S = p.s[q.s];
            return S.T + ((size_t)q.kt * S.nb * 8 + (size_t)(q.bg - S.nb0) * 8) * TW;
        };
        auto src_x = [&](const Cur& q) -> const uint32_t* {
            return reinterpret_cast<const uint32_t*>(p.xh + ((size_t)q.s * p.KT + q.kt) * (size_t)(2 * MP * 8));
        };
        constexpr int WP = UNIT_W / 4;                 // 16-byte pieces of a unit's tiles
        constexpr int XP = SLICE_W / 4;                // ... of its activation slice
        auto fill = [&](int i, int slot, bool w, bool x, Cur& q) {
            const uint32_t st = sbase + (uint32_t)slot * (STAGE_W * 4);
            const int m = min(UPS, n - i * UPS);
            if constexpr (BULKW) {   // weights only (fused path): lane 0 announces this producer's bytes and copies
                const int mine = m > pw ? (m - pw + PRODUCERS - 1) / PRODUCERS : 0;
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)(mine * UNIT_W * 4));
                for (int j = pw; j < m; j += PRODUCERS, step2(q))
                    if (lane == 0) bulk_g2s(st + j * UNIT_W * 4, src_w(q), UNIT_W * 4, &full[slot]);
                return;
            }
            for (int j = pw; j < m; j += PRODUCERS, step2(q)) {
                if (w) {
                    const uint32_t* src = src_w(q);
#pragma unroll
                    for (int k = lane; k < WP; k += 32) cp_async16_sa(st + (j * UNIT_W + k * 4) * 4, src + k * 4);
                }
                if (x) {
                    const uint32_t* src = src_x(q);
                    for (int k = lane; k < XP; k += 32)
                        cp_async16_sa(st + (UPS * UNIT_W + j * SLICE_W + k * 4) * 4, src + k * 4);
                }
            }
        };
        Cur cur = start();
        const int pre = min(nst, p.stages);
        if constexpr (FUSED) {
            for (int i = 0; i < pre; ++i) {
                fill(i, i, true, false, cur);
                if (!BULKW) cp_async_arrive(&full[i]);
            }
        } else {
            // weights do not depend on the previous kernel: fetch them first, then (after the wait) the activations
            Cur c0 = cur;
            for (int i = 0; i < pre; ++i) fill(i, i, true, false, cur);
            pdl_wait();
            for (int i = 0; i < pre; ++i) {
                fill(i, i, false, true, c0);
                cp_async_arrive(&full[i]);
            }
        }
        for (int i = p.stages, slot = 0, phase = 0; i < nst; ++i) {
            if (!mbar_wait(&empty[slot], phase)) break;   // gave up (status recorded)
            fill(i, slot, true, !FUSED, cur);
            if (!BULKW) cp_async_arrive(&full[slot]);
            if (++slot == p.stages) {
                slot = 0;
                phase ^= 1;
            }
        }
    } else {

        // ---------- consumers: warp w decodes tile w of every unit; even and odd units into separate sums ----------
        const int g = lane >> 2, t = lane & 3;
        const int grp = warp >> 3, wl = warp & 7;
        constexpr int CT = CWARPS * 32;

        float acc[2][NTG][4];
    #pragma unroll
        for (int e = 0; e < 2; ++e)
    #pragma unroll
            for (int q = 0; q < NTG; ++q) acc[e][q][0] = acc[e][q][1] = acc[e][q][2] = acc[e][q][3] = 0.f;

        if constexpr (FUSED) {   // rows >= M of the rotated activations are zero once and for all
            const int words = p.xh_chunks * 8 * SLICE_W;
            for (int i = threadIdx.x; i < words; i += CT) xrot[i] = 0u;
            named_sync(1, CT);
        }
        int bg = bg0, kt = kt0, li = 0, j = 0, slot = 0, phase = 0;
        bool from_zero = kt0 == 0;     // the current segment starts at the block's first k-tile
        int chunk0 = 0;                // fused: first 128-input chunk held in xrot
        bool seg_start = true;
        auto advance = [&]() {
            if (++slot == p.stages) {
                slot = 0;
                phase ^= 1;
            }
        };
        auto rotate_segment = [&]() {  // rotate the current segment's inputs (from unit li on) into shared memory
            const int seg_kt1 = min(p.KT, kt + (n - li));
            chunk0 = kt >> 3;
            const int nch = ((seg_kt1 + 7) >> 3) - chunk0;
            rotate_items<MP>(p, p.s[shard_of(bg, p)].suh, chunk0, nch, warp, lane, reinterpret_cast<__half*>(xrot));
            named_sync(1, CT);
            seg_start = false;
        };
        // Segment end: this warp's 16 columns (even + odd sums) into red[token][column], then by the segment's place
        // in its block: the whole block (finish in place), a later k-slice (store the tagged partial: it is this
        // CTA's first segment), or the block's first k-slice with the block running on past this CTA's range (the
        // finisher: its last segment).
        auto segment_end = [&]() {
            const int col = wl * 16 + g;
    #pragma unroll
            for (int gi = 0; gi < GROUPS; ++gi) {     // group 0's sums, then group 1's added, in that order
                if (gi == grp) {
    #pragma unroll
                    for (int q = 0; q < NTG; ++q) {
                        const int r0 = 8 * q + 2 * t;
                        float* rr = red + r0 * RED_STRIDE + col;
                        const float v0 = acc[0][q][0] + acc[1][q][0], v1 = acc[0][q][1] + acc[1][q][1];
                        const float v2 = acc[0][q][2] + acc[1][q][2], v3 = acc[0][q][3] + acc[1][q][3];
                        if (gi == 0) {
                            rr[0] = v0; rr[RED_STRIDE] = v1; rr[8] = v2; rr[RED_STRIDE + 8] = v3;
                        } else {
                            rr[0] += v0; rr[RED_STRIDE] += v1; rr[8] += v2; rr[RED_STRIDE + 8] += v3;
                        }
                    }
                }
                if (GROUPS > 1 && gi + 1 < GROUPS) named_sync(1, CT);
            }
            named_sync(1, CT);

            const DShard& S = p.s[shard_of(bg, p)];
            const int bl = bg - S.nb0;
            if (from_zero && kt == p.KT) {   // this CTA owns the whole block: finish it now
                const uint2 sv = load_svh(S, bl, lane);
                for (int r = warp; r < p.M; r += CWARPS) {
                    const float4 q = *reinterpret_cast<const float4*>(red + r * RED_STRIDE + 4 * lane);
                    float v[4] = {q.x, q.y, q.z, q.w};
                    finish_store(v, lane, S, bl, r, p, sv);
                }
            } else if (p.S > 1) {            // partial of a clustered block: stays in red, added after the loop
            } else {
                // equal k-slices: slice j stores the rows it does not finish and finishes the rows r = j (mod S), so
                // the S CTAs of a block share the finishing; otherwise a later k-slice stores its whole partial and the
                // CTA holding the block's first k-tile (its last segment) finishes every row
                const int nsl = p.kslices, j = nsl > 1 ? c % nsl : 0;
                const bool fin = nsl > 1 || from_zero;
                if (nsl > 1 || !from_zero) store_partial(p, red, c, warp, lane, [&](int r) { return nsl > 1 && r % nsl == j; });
                if (fin) {
                    const int c0 = c - j, n = nsl > 1 ? nsl : cta_of(bg * p.KT + p.KT - 1, p) - c + 1;
                    const int step = nsl > 1 ? nsl : 1;
                    const uint2 sv = load_svh(S, bl, lane);
                    for (int r = j + step * warp; r < p.M; r += step * CWARPS) finish_row(p, red, c0, n, j, r, S, bl, sv, lane);
                }
            }
            named_sync(1, CT);   // red (and the rotation buffer) are reused by the next segment
    #pragma unroll
            for (int e = 0; e < 2; ++e)   // zeroed here, not above: dead, not zero, while the block is finished
    #pragma unroll
                for (int q = 0; q < NTG; ++q) acc[e][q][0] = acc[e][q][1] = acc[e][q][2] = acc[e][q][3] = 0.f;
            if (kt == p.KT) {
                kt = 0;
                ++bg;
                from_zero = true;
            }
            seg_start = true;
        };

        // Decode ahead: the weights are not the previous kernel's output, so units are decoded into shared memory
        // (pre) before the wait on that kernel, while this CTA would otherwise sit idle: all of them (ahead_all), or
        // the first npre (whole stages of this CTA's one segment). Their products follow the wait in the loop's own
        // order and accumulators, so the sums are the bits the loop gives without decoding ahead.
        const bool ah = FUSED && p.ahead_all;
        if constexpr (FUSED) {
            const int nahead = ah ? nst : p.npre / UPS;
            for (int sidx = 0; sidx < nahead; ++sidx) {
                mbar_wait(&full[slot], phase);
                const uint32_t* st = smem + (size_t)slot * STAGE_W;
                const int m = min(UPS, n - sidx * UPS);
    #pragma unroll
                for (int j2 = 0; j2 < UPS / GROUPS; ++j2) {
                    const int jj = j2 * GROUPS + grp;
                    if (jj < m) {
                        uint32_t a[4];
                        decode_a<CB, K>(st + jj * UNIT_W + wl * TW, lane, a);
                        pre[((sidx * UPS + jj) * 8 + wl) * 32 + lane] = make_uint4(a[0], a[1], a[2], a[3]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                advance();
            }
        }
        pdl_wait();
        if constexpr (FUSED) {
            if (!ah && p.npre) {
                rotate_segment();
                for (int sidx = 0; sidx < p.npre / UPS; ++sidx) {
    #pragma unroll
                    for (int j2 = 0; j2 < UPS / GROUPS; ++j2) {
                        const int jj = j2 * GROUPS + grp;
                        const uint4 v = pre[((sidx * UPS + jj) * 8 + wl) * 32 + lane];
                        const uint32_t a[4] = {v.x, v.y, v.z, v.w};
                        const uint32_t* xs = xrot + (size_t)(kt + sidx * UPS + jj - 8 * chunk0) * SLICE_W;
    #pragma unroll
                        for (int q = 0; q < NTG; ++q)
                            mma16816(acc[j2 & 1][q], a, xs[(8 * q + g) * 4 + t], xs[(MP + 8 * q + g) * 4 + t]);
                    }
                }
                kt += p.npre;
                li = p.npre;
            }
        }
        while (li < n) {
            if (FUSED && seg_start) rotate_segment();   // rotate this segment's inputs into shared memory
            if (j == 0 && !ah) mbar_wait(&full[slot], phase);
            const uint32_t* st = smem + (size_t)slot * STAGE_W;
            const int stage_n = min(UPS, n - (li - j));
            const int run_end = min(stage_n, j + (p.KT - kt));
            const int kt_at_j = kt, u_at_0 = li - j;   // u_at_0: this stage's first unit in the CTA's range
            auto slice = [&](int jj) -> const uint32_t* {
                if constexpr (FUSED) return xrot + (size_t)(kt_at_j + jj - j - 8 * chunk0) * SLICE_W;
                else return st + UPS * UNIT_W + jj * SLICE_W;
            };
            auto tile = [&](int jj, uint32_t (&a)[4]) {   // unit jj of the stage: decoded ahead, or decoded now
                if (ah) {
                    const uint4 v = pre[((u_at_0 + jj) * 8 + wl) * 32 + lane];
                    a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
                } else {
                    decode_a<CB, K>(st + jj * UNIT_W + wl * TW, lane, a);
                }
            };
            if (j == 0 && run_end == UPS) {      // the common case: a whole stage inside one segment
    #pragma unroll
                for (int j2 = 0; j2 < UPS / GROUPS; ++j2) {
                    const int jj = j2 * GROUPS + grp;
                    uint32_t a[4];
                    tile(jj, a);
                    const uint32_t* xs = slice(jj);
    #pragma unroll
                    for (int q = 0; q < NTG; ++q)
                        mma16816(acc[j2 & 1][q], a, xs[(8 * q + g) * 4 + t], xs[(MP + 8 * q + g) * 4 + t]);
                }
            } else {
                for (int jj = j; jj < run_end; ++jj) {
                    if (GROUPS > 1 && (jj % GROUPS) != grp) continue;
                    uint32_t a[4];
                    tile(jj, a);
                    const uint32_t* xs = slice(jj);
    #pragma unroll
                    for (int q = 0; q < NTG; ++q) mma16816(acc[0][q], a, xs[(8 * q + g) * 4 + t], xs[(MP + 8 * q + g) * 4 + t]);
                }
            }
            kt += run_end - j;
            li += run_end - j;
            j = run_end;
            if (j == stage_n) {
                if (!ah) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                    advance();
                }
                j = 0;
            }
            if (kt != p.KT && li != n) continue;
            segment_end();
        }
    }

    if (p.S > 1) {   // the block's S CTAs (one cluster, rank = k-slice) add their partials in rank order
        cluster_sync_all();
        if (warp < CWARPS) {
            const int rank = (int)cluster_rank();
            const DShard& Sd = p.s[shard_of(bg0, p)];
            const int bl = bg0 - Sd.nb0;
            const uint2 sv = load_svh(Sd, bl, lane);
            for (int r = rank + p.S * warp; r < p.M; r += p.S * CWARPS) {
                const float* rr = red + r * RED_STRIDE + 4 * lane;
                float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int q = 0; q < p.S; ++q) {
                    const float4 v = ld_cluster_f4(rr, (uint32_t)q);
                    sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
                }
                float v4[4] = {sum.x, sum.y, sum.z, sum.w};
                finish_store(v4, lane, Sd, bl, r, p, sv);
            }
        }
        cluster_sync_all();   // no CTA leaves while another still reads its shared memory
    }
}

// ------------------------------------------------------------------------------------------------------------------
// dequant (experts_grouped.cuh:321-340): one warp a tile, exact reference values
// ------------------------------------------------------------------------------------------------------------------
template <int CB, int K>
__global__ void __launch_bounds__(128) dequant_kernel(const uint32_t* __restrict__ T, __half* __restrict__ out,
                                                      int KT, int NT) {
    const int tile = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (tile >= KT * NT) return;
    const int kt = tile / NT, nt = tile % NT, N = NT * 16;
    uint32_t st[8];
    tile_states<K>(T + (size_t)tile * 8 * K, lane, st);
    const uint32_t v[4] = {cb_exact<CB>(st[0], st[1]), cb_exact<CB>(st[2], st[3]), cb_exact<CB>(st[4], st[5]),
                           cb_exact<CB>(st[6], st[7])};
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __half2 h = u2h(v[q]);
        const int col = nt * 16 + g + 8 * (q >> 1);
        const int row = kt * 16 + 2 * t + 8 * (q & 1);
        out[(size_t)row * N + col] = __low2half(h);
        out[(size_t)(row + 1) * N + col] = __high2half(h);
    }
}

// y = fp16(H(x * pre) / sqrt(128) * post) (dense.cu:242-265)
__global__ void __launch_bounds__(128) had_kernel(const __half* __restrict__ x, const __half* __restrict__ pre,
                                                  const __half* __restrict__ post, __half* y, int K) {
    const int blk = blockIdx.x * 4 + (threadIdx.x >> 5), row = blockIdx.y, lane = threadIdx.x & 31;
    if (blk * 128 >= K) return;
    const size_t i = (size_t)row * K + blk * 128 + 4 * lane;
    float v[4];
    load4(x, F16, i, v);
    if (pre) {
        float s[4];
        load4(pre, F16, blk * 128 + 4 * lane, s);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(v[j], s[j]);
    }
    fwht128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= HAD_SCALE;
    if (post) {
        float s[4];
        load4(post, F16, blk * 128 + 4 * lane, s);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] *= s[j];
    }
    store4(y, F16, i, v);
}

size_t dense_smem_bytes(int K, int ntg, bool fused, int chunks, int npre, int stages = STAGES) {
    const int tw = 8 * K, unit_w = 8 * tw, slice_w = 8 * ntg * 8;
    return (size_t)stages * UPS * (unit_w + (fused ? 0 : slice_w)) * 4 + (size_t)8 * ntg * RED_STRIDE * 4 +
           (fused ? (size_t)chunks * 8 * slice_w * 4 + (size_t)npre * 8 * 32 * 16 : 0) + 2 * STAGES * 8;
}

// dynamic shared memory a CTA may take: most of an SM's 227 KB with one resident CTA an SM, half of it with two
constexpr size_t SMEM_LIMIT = (RESIDENT == 1 ? 220 : 110) * 1024;

// ESPALIER_DENSE_AHEAD=0 turns the decode ahead of the launch wait off (for comparison); on by default.
bool ahead_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("ESPALIER_DENSE_AHEAD");
        return !(v && v[0] == '0');
    }();
    return on;
}

// With fewer blocks than SMs the default gives every block S = SMs / blocks equal k-slices (one segment a CTA,
// G = blocks * S CTAs). ESPALIER_DENSE_SPLIT=ranges splits the units in one equal range an SM instead (every SM busy,
// a CTA meeting at most two blocks), when every CTA's units fit the shared memory decoded: measured slower (0.87 vs
// 0.80 ms for 40 config-2 blocks at batch 1, 1.76 vs 1.55 ms at 32 rows), a CTA's second segment adding its own
// rotation, reduction and partial after the launch wait.
bool split_ranges() {
    static const bool on = [] {
        const char* v = std::getenv("ESPALIER_DENSE_SPLIT");
        return v && std::strcmp(v, "ranges") == 0;
    }();
    return on;
}

// ESPALIER_DENSE_CLUSTER=1 finishes split blocks inside a thread-block cluster (DSMEM reads of the k-slices' partials)
// instead of through global partials. Off by default: on the config-2 block it measured slower (1.09 vs 0.84 ms for
// 40 blocks at batch 1), the cluster launches costing more in scheduling and in overlap with the previous launch than
// the shorter finishing saves.
bool cluster_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("ESPALIER_DENSE_CLUSTER");
        return v && v[0] == '1';
    }();
    return on;
}

template <int CB, int K, int NTG, bool FUSED>
int launch_dense(DenseParams p, void* stream) {
    auto kern = dense_kernel<CB, K, NTG, FUSED>;
    const size_t smem = dense_smem_bytes(K, NTG, FUSED, p.xh_chunks, FUSED ? p.npre : 0, p.stages);
    static size_t opted = 0;
    if (smem > opted) {
        if (int rc = allow_smem(kern, FUSED ? SMEM_LIMIT : smem)) return rc;
        opted = FUSED ? SMEM_LIMIT : smem;
    }
    if (p.S > 1) {   // one cluster a block, if at least one such cluster fits on the device
        static bool nonportable = false;
        if (p.S > 8 && !nonportable) {
            if (cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributeNonPortableClusterSizeAllowed,
                                     1) != cudaSuccess) {
                cudaGetLastError();
                p.S = 0;
            } else {
                nonportable = true;
            }
        }
        if (p.S > 1) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(p.G);
            cfg.blockDim = dim3(THREADS);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = static_cast<unsigned>(p.S);
            at[0].val.clusterDim.y = at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
                cudaGetLastError();
                p.S = 0;
            }
        }
    }
    if (p.S > 1) return launch_cluster(kern, dim3(p.G), dim3(THREADS), smem, stream, true, p.S, p);
    return launch(kern, dim3(p.G), dim3(THREADS), smem, stream, true, p);
}

template <int CB, int K>
int launch_dense_ntg(const DenseParams& p, bool fused, void* stream) {
    // the fused path is planned for one token group only (up to 8 rows)
    if (fused) return p.Mp == 8 ? launch_dense<CB, K, 1, true>(p, stream) : ESP_ERR_INVALID;
    switch (p.Mp / 8) {
        case 1: return launch_dense<CB, K, 1, false>(p, stream);
        case 2: return launch_dense<CB, K, 2, false>(p, stream);
        case 3: return launch_dense<CB, K, 3, false>(p, stream);
        default: return launch_dense<CB, K, 4, false>(p, stream);
    }
}

// Everything esp_dense checks and derives on the host, before any device work.
struct DensePlan {
    DenseParams p;
    RotParams r;
    bool fused;
    int K;
    int cb;
};

int dense_plan(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats, int n_mats,
               int k2, int cb, void* y, int y_dtype, long long y_stride, void* xh, size_t xh_bytes, float* z,
               size_t z_bytes, int* counters, int n_counters, DensePlan& pl) {
    ESP_REQUIRE(x && y && mats && xh && counters, ESP_ERR_INVALID, "esp_dense: null pointer");
    ESP_REQUIRE(n_mats >= 1 && n_mats <= MAX_SHARDS, ESP_ERR_INVALID, "esp_dense: 1 to 4 matrices a launch");
    ESP_REQUIRE(m >= 1 && m <= 32, ESP_ERR_INVALID, "esp_dense: 1 to 32 rows");
    ESP_REQUIRE(k >= 128 && k % 128 == 0, ESP_ERR_INVALID, "esp_dense: K must be a positive multiple of 128");
    ESP_REQUIRE(k2 % 2 == 0 && case_supported(cb, k2 / 2), ESP_ERR_UNSUPPORTED,
                "esp_dense: unsupported codebook/width: cb=%d k2=%d", cb, k2);
    ESP_REQUIRE(x_dtype >= 0 && x_dtype <= 2 && y_dtype >= 0 && y_dtype <= 2, ESP_ERR_INVALID, "esp_dense: dtype");
    ESP_REQUIRE(x_stride >= k && aligned(x, 16) && (x_stride * (x_dtype == F32 ? 4 : 2)) % 8 == 0, ESP_ERR_INVALID,
                "esp_dense: x rows must be 8-byte aligned with a stride >= K");
    const int K = k2 / 2;
    pl = DensePlan{};
    pl.K = K;
    pl.cb = cb;
    DenseParams& p = pl.p;
    RotParams& r = pl.r;
    int nbt = 0;
    for (int s = 0; s < n_mats; ++s) {
        const esp_matrix_t& mt = mats[s];
        ESP_REQUIRE(mt.trellis && mt.suh && mt.svh, ESP_ERR_INVALID, "esp_dense: matrix %d has a null pointer", s);
        ESP_REQUIRE(mt.n >= 128 && mt.n % 128 == 0, ESP_ERR_INVALID, "esp_dense: matrix %d: N must be a multiple of 128",
                    s);
        ESP_REQUIRE(aligned(mt.trellis, 16) && aligned(mt.suh, 8) && aligned(mt.svh, 8), ESP_ERR_INVALID,
                    "esp_dense: matrix %d: misaligned tensor", s);
        ESP_REQUIRE(mt.col0 >= 0 && mt.col0 % 4 == 0 && mt.col0 + mt.n <= y_stride, ESP_ERR_INVALID,
                    "esp_dense: matrix %d columns past y", s);
        p.s[s] = DShard{reinterpret_cast<const uint32_t*>(mt.trellis), reinterpret_cast<const __half*>(mt.suh),
                        reinterpret_cast<const __half*>(mt.svh), nbt, mt.n / 128, mt.col0};
        r.suh[s] = reinterpret_cast<const __half*>(mt.suh);
        nbt += mt.n / 128;
    }
    ESP_REQUIRE(n_counters >= nbt, ESP_ERR_SCRATCH, "esp_dense: counters need %d entries, got %d", nbt, n_counters);
    ESP_REQUIRE(xh_bytes >= esp_dense_xh_bytes(m, k, n_mats) && aligned(xh, 16), ESP_ERR_SCRATCH,
                "esp_dense: xh scratch needs %zu bytes, got %zu", esp_dense_xh_bytes(m, k, n_mats), xh_bytes);
    const int mp = (m + 7) / 8 * 8;
    p.n = n_mats;
    p.xh = static_cast<const __half*>(xh);
    p.y = y;
    p.y_dtype = y_dtype;
    p.y_stride = y_stride;
    p.counters = counters;
    p.M = m;
    p.Mp = mp;
    p.K = k;
    p.KT = k / 16;
    p.U = nbt * p.KT;
    p.NB = nbt;
    const int sms = device_sms() * CTAS_PER_SM;
    // the fused path rotates each segment's inputs inside the kernel; a segment spans at most the CTA's units or one
    // block's k-tiles, plus one chunk of misalignment
    auto chunks_for = [&](int G) {
        const long long per_cta = (p.U + G - 1) / G;
        const int max_kt = (int)std::min<long long>(p.KT, per_cta);
        return std::min(p.KT / 8, (max_kt + 7) / 8 + 1);
    };
    // the deepest ring (down to 3 stages) beside all of a CTA's units decoded, or 0 if none fits
    auto ahead_stages = [&](int G) {
        const int nmax = (p.U + G - 1) / G;
        for (int st = STAGES; st >= 3; --st)
            if (dense_smem_bytes(K, 1, true, chunks_for(G), nmax, st) <= SMEM_LIMIT) return st;
        return 0;
    };
    // Fewer blocks than SMs: S CTAs a block, each an equal k-slice (one segment a CTA, a block's S partials), or with
    // split_ranges one equal range of units an SM when every CTA's units fit the shared memory decoded. Otherwise one
    // range an SM over whole blocks, with at most a partial block at each end. The choice depends on the shape alone
    // (not on the rows), so a row's bits do not depend on the others.
    const bool few = nbt < sms;
    p.G = few ? nbt * std::min(sms / nbt, p.KT) : sms;
    if (few && split_ranges() && !cluster_enabled() && ahead_stages(std::min(sms, p.U))) p.G = std::min(sms, p.U);
    ESP_REQUIRE((long long)p.U * p.G < (1ll << 31), ESP_ERR_INVALID, "esp_dense: layer too large (%d units)", p.U);
    // k-slices of a block finish inside one thread-block cluster when there are 2..16 of them (the limit of a
    // non-portable cluster on this GPU)
    p.S = (few && p.G % nbt == 0 && cluster_enabled() && p.G / nbt >= 2 && p.G / nbt <= 16) ? p.G / nbt : 0;
    // above 8 rows a block's finishing is shared by its k-slices (measured: 1.20 vs 1.55 ms a 40-block step at 32
    // rows); up to 8 rows the first slice finishes alone (0.80 vs 0.81 ms at 1 row, 0.90 vs 1.01 ms at 8 rows)
    p.kslices = (few && p.G % nbt == 0 && p.G / nbt >= 2 && m > 8) ? p.G / nbt : 0;
    p.scale = cb_step(cb);
    p.Z = reinterpret_cast<uint64_t*>(z);
    const size_t zneed = (size_t)p.G * m * 128 * 8;
    ESP_REQUIRE((zneed == 0 || z) && z_bytes >= zneed && aligned(z, 16), ESP_ERR_SCRATCH,
                "esp_dense: Z scratch needs %zu bytes, got %zu", zneed, z_bytes);

    const int chunks = chunks_for(p.G);
    // up to 8 rows the in-kernel rotation is cheaper than a rotation launch; above, its loads serialise per row
    pl.fused = mp == 8 && dense_smem_bytes(K, mp / 8, true, chunks, 0) <= SMEM_LIMIT;
    // decode ahead (fused path, fewer blocks than CTAs): all of every CTA's units where they fit beside a ring of at
    // least 3 stages, else (the slices) as many whole stages of the one segment as the shared memory beside the ring
    // holds, leaving the loop at least one unit of every CTA (U / G is the smallest range)
    p.npre = 0;
    p.ahead_all = 0;
    p.stages = STAGES;
    if (pl.fused && few && ahead_enabled()) {
        if (const int st = p.S == 0 ? ahead_stages(p.G) : 0) {
            p.stages = st;
            p.ahead_all = 1;
            p.npre = (p.U + p.G - 1) / p.G;
        } else if (p.G % nbt == 0) {
            const size_t base = dense_smem_bytes(K, 1, true, chunks, 0);
            const int cap = base < SMEM_LIMIT ? (int)((SMEM_LIMIT - base) / (8 * 32 * 16)) : 0;
            p.npre = std::max(0, std::min(cap, p.U / p.G - 1) / UPS * UPS);
        }
    }
    p.x = x;
    p.x_dtype = x_dtype;
    p.x_stride = x_stride;
    p.xh_chunks = pl.fused ? chunks : 0;
    if (!pl.fused) {
        r.x = x;
        r.x_dtype = x_dtype;
        r.x_stride = x_stride;
        r.xh = static_cast<__half*>(xh);
        r.M = m;
        r.Mp = mp;
        r.K = k;
        r.KT = k / 16;
    }
    return ESP_OK;
}

int dense_run(const DensePlan& pl, void* stream) {
    if (!pl.fused) {
        const RotParams& r = pl.r;
        if (int rc = launch(rot_kernel, dim3((r.K / 128 + 3) / 4, r.Mp, pl.p.n), dim3(128), 0, stream, true, r))
            return rc;
    }
    int rc = ESP_ERR_UNSUPPORTED;
    switch (pl.cb * 16 + pl.K) {
#define ESP_DENSE_CASE(CB_, K_) \
    case CB_ * 16 + K_: rc = launch_dense_ntg<CB_, K_>(pl.p, pl.fused, stream); break;
        ESP_FOR_EACH_CASE(ESP_DENSE_CASE)
#undef ESP_DENSE_CASE
        default: return set_error(ESP_ERR_UNSUPPORTED, "esp_dense: unsupported codebook/width: cb=%d K=%d", pl.cb, pl.K);
    }
    if (rc) return rc;
    return ok();
}

}  // namespace
}  // namespace esp

using namespace esp;

extern "C" {

size_t esp_dense_xh_bytes(int m, int k, int n_mats) {
    const int mp = (m + 7) / 8 * 8;
    return (size_t)n_mats * mp * k * 2;
}

size_t esp_dense_z_bytes(int m) { return (size_t)device_sms() * CTAS_PER_SM * m * 128 * 8; }

int esp_dense(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats, int n_mats,
              int k2, int cb, void* y, int y_dtype, long long y_stride, void* xh, size_t xh_bytes, float* z,
              size_t z_bytes, int* counters, int n_counters, void* stream) {
    DensePlan pl;
    if (int rc = dense_plan(x, x_dtype, x_stride, m, k, mats, n_mats, k2, cb, y, y_dtype, y_stride, xh, xh_bytes, z,
                            z_bytes, counters, n_counters, pl))
        return rc;
    return dense_run(pl, stream);
}

int esp_dequant(const int16_t* trellis, int kin, int n, int k2, int cb, uint16_t* out, void* stream) {
    ESP_REQUIRE(trellis && out, ESP_ERR_INVALID, "esp_dequant: null pointer");
    ESP_REQUIRE(kin > 0 && n > 0 && kin % 16 == 0 && n % 16 == 0, ESP_ERR_INVALID, "esp_dequant: shape %dx%d", kin, n);
    ESP_REQUIRE(aligned(trellis, 4) && aligned(out, 2), ESP_ERR_INVALID, "esp_dequant: misaligned pointer");
    ESP_REQUIRE(k2 % 2 == 0 && case_supported(cb, k2 / 2), ESP_ERR_UNSUPPORTED,
                "no instance for codebook %d K2 %d", cb, k2);
    const int KT = kin / 16, NT = n / 16;
    const dim3 grid((unsigned)((KT * NT + 3) / 4));
    const uint32_t* T = reinterpret_cast<const uint32_t*>(trellis);
    __half* o = reinterpret_cast<__half*>(out);
    int rc = ESP_ERR_UNSUPPORTED;
    switch (cb * 16 + k2 / 2) {
#define ESP_DQ_CASE(CB_, K_) \
    case CB_ * 16 + K_: rc = launch(dequant_kernel<CB_, K_>, grid, dim3(128), 0, stream, false, T, o, KT, NT); break;
        ESP_FOR_EACH_CASE(ESP_DQ_CASE)
#undef ESP_DQ_CASE
        default: break;
    }
    if (rc) return rc;
    return ok();
}

int esp_had(const uint16_t* x, int m, int k, const uint16_t* pre, const uint16_t* post, uint16_t* y, void* stream) {
    ESP_REQUIRE(x && y, ESP_ERR_INVALID, "esp_had: null pointer");
    ESP_REQUIRE(m >= 0 && k > 0 && k % 128 == 0, ESP_ERR_INVALID, "had: K must be a multiple of 128");
    ESP_REQUIRE(aligned(x, 8) && aligned(y, 8) && (!pre || aligned(pre, 8)) && (!post || aligned(post, 8)),
                ESP_ERR_INVALID, "esp_had: misaligned pointer");
    if (m == 0) return ok();
    if (int rc = launch(had_kernel, dim3((k / 128 + 3) / 4, m), dim3(128), 0, stream, false,
                        reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(pre),
                        reinterpret_cast<const __half*>(post), reinterpret_cast<__half*>(y), k))
        return rc;
    return ok();
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------------------
// Allocation-free dense layer. Some callers cannot allocate device memory at the moment they run a layer: a serving
// engine that has already handed nearly all of HBM to its KV cache, host code bound only through this C ABI with no
// allocator of its own, or a path that must not take cudaMalloc's implicit device synchronisation. For them this entry
// point keeps the dense kernel's scratch (rotated activations, split-K partial sums, arrival counters) in one fixed
// array of device memory that every GPU loading this library holds until the process exits.
// ------------------------------------------------------------------------------------------------------------------
namespace esp {
namespace {
constexpr int NOALLOC_MAX_K = 4096;            // input features
constexpr int NOALLOC_MAX_BLOCKS = 8192;       // 128-column blocks of all matrices of one call (1,048,576 columns)
constexpr int NOALLOC_MAX_SMS = 160;
// tagged partial sums: one slot a CTA (CTAS_PER_SM a streaming multiprocessor) x 32 rows x 128 columns x 8 bytes;
// zero at load (static storage) and left zero by every call that completes
constexpr size_t NOALLOC_Z = (size_t)NOALLOC_MAX_SMS * CTAS_PER_SM * 32 * 128 * 8;
constexpr size_t NOALLOC_XH = (size_t)MAX_SHARDS * 32 * NOALLOC_MAX_K * 2;
constexpr size_t NOALLOC_CNT = (size_t)NOALLOC_MAX_BLOCKS * 4;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_Z + NOALLOC_XH + NOALLOC_CNT];   // 6.0 MiB

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};

// The array's device address for the current device, looked up once per device (its name in host code is only a
// host-side stand-in). Returns nullptr after recording the error.
unsigned char* noalloc_scratch() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        set_error(ESP_ERR_CUDA, "esp_dense_noalloc: no current device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr) {
            set_error(ESP_ERR_CUDA, "esp_dense_noalloc: scratch address: %s", cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_addr[dev] = ptr;
    }
    return static_cast<unsigned char*>(g_noalloc_addr[dev]);
}
}  // namespace
}  // namespace esp

extern "C" int esp_dense_noalloc(const void* x, int x_dtype, long long x_stride, int m, int k,
                                 const esp_matrix_t* mats, int n_mats, int k2, int cb, void* y, int y_dtype,
                                 long long y_stride, void* stream) {
    using namespace esp;
    ESP_REQUIRE(mats && n_mats >= 1 && n_mats <= MAX_SHARDS, ESP_ERR_INVALID, "esp_dense_noalloc: 1 to 4 matrices");
    long long cols = 0;
    for (int s = 0; s < n_mats; ++s) cols += mats[s].n;
    ESP_REQUIRE(k <= NOALLOC_MAX_K, ESP_ERR_INVALID,
                "esp_dense_noalloc: K=%d exceeds the static scratch limit of %d inputs", k, NOALLOC_MAX_K);
    ESP_REQUIRE(cols <= (long long)NOALLOC_MAX_BLOCKS * 128, ESP_ERR_INVALID,
                "esp_dense_noalloc: %lld output columns exceed the static scratch limit of %d", cols,
                NOALLOC_MAX_BLOCKS * 128);
    ESP_REQUIRE(device_sms() <= NOALLOC_MAX_SMS, ESP_ERR_INVALID,
                "esp_dense_noalloc: %d SMs exceed the static scratch limit of %d", device_sms(), NOALLOC_MAX_SMS);
    unsigned char* base = noalloc_scratch();
    if (!base) return ESP_ERR_CUDA;
    float* z = reinterpret_cast<float*>(base);
    void* xh = base + NOALLOC_Z;
    int* counters = reinterpret_cast<int*>(base + NOALLOC_Z + NOALLOC_XH);
    // every argument is checked before the shared array is touched: a rejected call leaves it as it was
    DensePlan pl;
    if (int rc = dense_plan(x, x_dtype, x_stride, m, k, mats, n_mats, k2, cb, y, y_dtype, y_stride, xh, NOALLOC_XH, z,
                            NOALLOC_Z, counters, NOALLOC_MAX_BLOCKS, pl))
        return rc;
    return dense_run(pl, stream);
}
