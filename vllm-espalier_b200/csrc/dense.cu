// Dense layer decode for 1..32 rows: every matrix of one layer (q/k/v, in_proj_qkv/z, o, the head) in one
// persistent launch that streams the compressed trellis once and decodes each weight once for all rows.
//
// Reference behaviour (vllm_espalier/csrc/dense.cu:130-238, ops.py, dense.py): y_s = H(H(x * suh_s) @ W_s) * svh_s
// written into columns col0_s of y, fp16 rotated activations, fp32 sums, output in the model's dtype; rows are
// independent, split and warp ranges depend on the shape alone, every sum runs in a fixed order.
//
// B200 design:
//   * rot_kernel writes fp16 H(x * suh_s) / sqrt(128) for every matrix once, in a tile-major layout
//     [s][k-tile][k-half][row][8] whose per-k-tile slice is one contiguous bulk copy (and bank-conflict free as an MMA
//     B fragment).
//   * dense_kernel: one CTA per SM. The layer is a list of units (128-column block, 16-row k-tile) in block-major
//     order, split into equal contiguous ranges, one per CTA (stream-K), so every SM decodes the same number of
//     weights. A producer warp streams each unit's 8 tiles (8K words each) and its activation slice into a ring of
//     shared-memory stages with cp.async.bulk (TMA) and mbarriers; 16 consumer warps (two groups of 8, alternating
//     k-tiles) decode one tile each per unit straight into the A fragment of mma.sync m16n8k16 (M = 16 output
//     columns, N = 8 tokens), i.e. the weights are decoded once whatever the number of rows.
//   * A block whose k range is split across CTAs is finished by the last CTA to arrive (atomic counter), which adds
//     the partial sums in CTA order; a block owned by one CTA is finished in place. Finishing = FWHT-128 of the sums,
//     * step, * H/sqrt(128) * svh, in the reference's order, then the store in y's dtype.
#include <cuda_runtime.h>

#include "common.cuh"
#include "host.hpp"
#include "trellis.cuh"

ESP_DEFINE_STATUS_READER(dense)

namespace esp {
namespace {

constexpr int MAX_SHARDS = 4;
constexpr int CWARPS = 16;                     // consumer warps (two groups of 8: one warp per tile of a unit)
constexpr int THREADS = (CWARPS + 1) * 32;     // + one producer warp
constexpr int UPS = 2;                         // units per pipeline stage
constexpr int RED_STRIDE = 132;                // fp32 row stride of the reduction buffer (bank-conflict free)

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
    const __half* xh;            // rotated activations [n][KT][2][Mp][8]
    void* y;
    int y_dtype;
    long long y_stride;
    float* Z;                    // partial sums [2 * G][M][128]
    int* counters;               // [blocks], zero on entry and on exit
    int M, Mp, K, KT, U, G;      // rows, padded rows, inputs, k tiles, units, CTAs
    int stages;                  // pipeline depth
    float scale;                 // codebook step of the kernel form
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

__device__ __forceinline__ long long range_start(int c, const DenseParams& p) {
    return (long long)c * p.U / p.G;
}
__device__ __forceinline__ int cta_of(long long u, const DenseParams& p) {
    return (int)(((u + 1) * p.G - 1) / p.U);
}

// The finished 4 outputs of lane `lane` of one row of a 128-column block (dense.cu:120-128) and their store.
__device__ __forceinline__ void finish_store(float (&v)[4], int lane, const DShard& S, int bl, int row,
                                             const DenseParams& p) {
    fwht128(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= p.scale;
    const __half* svh = S.svh + bl * 128 + 4 * lane;
    const uint2 sv = *reinterpret_cast<const uint2*>(svh);
    const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
    const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
    v[0] *= HAD_SCALE * s01.x; v[1] *= HAD_SCALE * s01.y; v[2] *= HAD_SCALE * s23.x; v[3] *= HAD_SCALE * s23.y;
    store4(p.y, p.y_dtype, (size_t)row * p.y_stride + S.col0 + bl * 128 + 4 * lane, v);
}

template <int CB, int K, int NTG>
__global__ void __launch_bounds__(THREADS, 1) dense_kernel(const __grid_constant__ DenseParams p) {
    constexpr int TW = 8 * K;                          // words a tile
    constexpr int UNIT_W = 8 * TW;                     // words a unit (8 tiles)
    constexpr int MP = 8 * NTG;
    constexpr int SLICE_W = MP * 8;                    // words of a unit's activation slice
    constexpr int STAGE_W = UPS * (UNIT_W + SLICE_W);
    extern __shared__ __align__(128) uint32_t smem[];
    uint32_t* stage_base = smem;                                        // [stages][STAGE_W]
    float* red = reinterpret_cast<float*>(smem + (size_t)p.stages * STAGE_W);   // [MP][RED_STRIDE]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + MP * RED_STRIDE);
    uint64_t* empty = full + p.stages;
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const long long u0 = range_start(c, p), u1 = range_start(c + 1, p);
    const int nunits = (int)(u1 - u0);
    const int nst = (nunits + UPS - 1) / UPS;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8 * UPS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == CWARPS) {   // ---------------- producer ----------------
        if (lane != 0) return;
        auto unit_src = [&](long long u, int& bytes) -> const uint32_t* {
            const int bg = (int)(u / p.KT), kt = (int)(u % p.KT);
            int s = 0;
#pragma unroll
            for (int i = 1; i < MAX_SHARDS; ++i)
                if (i < p.n && bg >= p.s[i].nb0) s = i;
            const DShard& S = p.s[s];
            bytes = UNIT_W * 4;
            return S.T + ((size_t)kt * (S.nb * 8) + (size_t)(bg - S.nb0) * 8) * TW;
        };
        auto slice_src = [&](long long u) -> const __half* {
            const int bg = (int)(u / p.KT), kt = (int)(u % p.KT);
            int s = 0;
#pragma unroll
            for (int i = 1; i < MAX_SHARDS; ++i)
                if (i < p.n && bg >= p.s[i].nb0) s = i;
            return p.xh + ((size_t)s * p.KT + kt) * (size_t)(2 * MP * 8);
        };
        auto issue = [&](int i, bool weights, bool acts) {
            const int slot = i % p.stages;
            uint32_t* st = stage_base + (size_t)slot * STAGE_W;
            for (int j = 0; j < UPS; ++j) {
                const long long u = u0 + (long long)i * UPS + j;
                if (u >= u1) break;
                int bytes;
                const uint32_t* src = unit_src(u, bytes);
                if (weights) bulk_g2s(st + j * UNIT_W, src, UNIT_W * 4, &full[slot]);
                if (acts) bulk_g2s(st + UPS * UNIT_W + j * SLICE_W, slice_src(u), SLICE_W * 4, &full[slot]);
            }
        };
        auto stage_bytes = [&](int i) -> uint32_t {
            const long long a = u0 + (long long)i * UPS;
            const int n = (int)min((long long)UPS, u1 - a);
            return (uint32_t)n * (UNIT_W + SLICE_W) * 4u;
        };
        const int pre = min(nst, p.stages);
        for (int i = 0; i < pre; ++i) {   // weights do not depend on the previous kernel: fetch them before waiting
            mbar_arrive_expect_tx(&full[i], stage_bytes(i));
            issue(i, true, false);
        }
        pdl_wait();
        for (int i = 0; i < pre; ++i) issue(i, false, true);
        for (int i = p.stages; i < nst; ++i) {
            const int slot = i % p.stages;
            if (!mbar_wait(&empty[slot], ((i / p.stages) - 1) & 1)) return;
            mbar_arrive_expect_tx(&full[slot], stage_bytes(i));
            issue(i, true, true);
        }
        return;
    }

    // -------------------- consumers: warp w = 8 * grp + wl decodes tile wl of the units of group grp --------------
    pdl_wait();
    const int grp = warp >> 3, wl = warp & 7;
    const int g = lane >> 2, t = lane & 3;
    constexpr int CT = CWARPS * 32;

    long long u = u0;
    while (u < u1) {
        const int bg = (int)(u / p.KT);
        const long long seg0 = u, seg1 = min(u1, (long long)(bg + 1) * p.KT);
        float acc[NTG][4];
#pragma unroll
        for (int q = 0; q < NTG; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;

        for (long long uu = seg0 + grp; uu < seg1; uu += 2) {
            const int li = (int)(uu - u0), stage = li / UPS, slot = stage % p.stages, j = li % UPS;
            mbar_wait(&full[slot], (stage / p.stages) & 1);
            const uint32_t* st = stage_base + (size_t)slot * STAGE_W;
            uint32_t a[4];
            decode_a<CB, K>(st + j * UNIT_W + wl * TW, lane, a);
            const uint32_t* xs = st + UPS * UNIT_W + j * SLICE_W;
#pragma unroll
            for (int q = 0; q < NTG; ++q) {
                const uint32_t b0 = xs[(8 * q + g) * 4 + t];
                const uint32_t b1 = xs[(MP + 8 * q + g) * 4 + t];
                mma16816(acc[q], a, b0, b1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- segment end: the two groups' sums, group 0 then group 1, into red[token][column] ----
        const int col = wl * 16 + g;
        if (grp == 0) {
#pragma unroll
            for (int q = 0; q < NTG; ++q) {
                const int r0 = 8 * q + 2 * t;
                red[r0 * RED_STRIDE + col] = acc[q][0];
                red[(r0 + 1) * RED_STRIDE + col] = acc[q][1];
                red[r0 * RED_STRIDE + col + 8] = acc[q][2];
                red[(r0 + 1) * RED_STRIDE + col + 8] = acc[q][3];
            }
        }
        named_sync(1, CT);
        if (grp == 1) {
#pragma unroll
            for (int q = 0; q < NTG; ++q) {
                const int r0 = 8 * q + 2 * t;
                red[r0 * RED_STRIDE + col] += acc[q][0];
                red[(r0 + 1) * RED_STRIDE + col] += acc[q][1];
                red[r0 * RED_STRIDE + col + 8] += acc[q][2];
                red[(r0 + 1) * RED_STRIDE + col + 8] += acc[q][3];
            }
        }
        named_sync(1, CT);

        int s = 0;
#pragma unroll
        for (int i = 1; i < MAX_SHARDS; ++i)
            if (i < p.n && bg >= p.s[i].nb0) s = i;
        const DShard& S = p.s[s];
        const int bl = bg - S.nb0;
        const bool complete = seg0 == (long long)bg * p.KT && seg1 == (long long)(bg + 1) * p.KT;
        if (complete) {
            for (int r = warp; r < p.M; r += CWARPS) {
                const float4 q = *reinterpret_cast<const float4*>(red + r * RED_STRIDE + 4 * lane);
                float v[4] = {q.x, q.y, q.z, q.w};
                finish_store(v, lane, S, bl, r, p);
            }
        } else {
            const long long first_bg = u0 / p.KT;
            const int slot = 2 * c + (bg == first_bg ? 0 : 1);
            float* zs = p.Z + (size_t)slot * p.M * 128;
            for (int r = warp; r < p.M; r += CWARPS)
                *reinterpret_cast<float4*>(zs + r * 128 + 4 * lane) =
                    *reinterpret_cast<const float4*>(red + r * RED_STRIDE + 4 * lane);
            __threadfence();
            named_sync(1, CT);
            const int c_lo = cta_of((long long)bg * p.KT, p), c_hi = cta_of((long long)(bg + 1) * p.KT - 1, p);
            if (threadIdx.x == 0) s_last = atomicAdd(&p.counters[bg], 1) == c_hi - c_lo;
            named_sync(1, CT);
            if (s_last) {
                __threadfence();
                for (int r = warp; r < p.M; r += CWARPS) {
                    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int cc = c_lo; cc <= c_hi; ++cc) {
                        const int sl = 2 * cc + ((long long)bg == range_start(cc, p) / p.KT ? 0 : 1);
                        const float4 q = __ldcg(reinterpret_cast<const float4*>(p.Z + ((size_t)sl * p.M + r) * 128 +
                                                                                4 * lane));
                        sum.x += q.x; sum.y += q.y; sum.z += q.z; sum.w += q.w;
                    }
                    float v[4] = {sum.x, sum.y, sum.z, sum.w};
                    finish_store(v, lane, S, bl, r, p);
                }
                if (threadIdx.x == 0) p.counters[bg] = 0;
            }
        }
        named_sync(1, CT);   // red is reused by the next segment
        u = seg1;
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

constexpr int STAGES = 8;

size_t dense_smem_bytes(int K, int ntg) {
    const int tw = 8 * K, unit_w = 8 * tw, slice_w = 8 * ntg * 8;
    return (size_t)STAGES * UPS * (unit_w + slice_w) * 4 + (size_t)8 * ntg * RED_STRIDE * 4 + 2 * STAGES * 8;
}

template <int CB, int K, int NTG>
int launch_dense(const DenseParams& p, void* stream) {
    auto kern = dense_kernel<CB, K, NTG>;
    const size_t smem = dense_smem_bytes(K, NTG);
    static bool opted = false;
    if (!opted) {
        if (int rc = allow_smem(kern, smem)) return rc;
        opted = true;
    }
    return launch(kern, dim3(p.G), dim3(THREADS), smem, stream, true, p);
}

template <int CB, int K>
int launch_dense_ntg(const DenseParams& p, void* stream) {
    switch (p.Mp / 8) {
        case 1: return launch_dense<CB, K, 1>(p, stream);
        case 2: return launch_dense<CB, K, 2>(p, stream);
        case 3: return launch_dense<CB, K, 3>(p, stream);
        default: return launch_dense<CB, K, 4>(p, stream);
    }
}

}  // namespace
}  // namespace esp

using namespace esp;

extern "C" {

size_t esp_dense_xh_bytes(int m, int k, int n_mats) {
    const int mp = (m + 7) / 8 * 8;
    return (size_t)n_mats * mp * k * 2;
}

size_t esp_dense_z_bytes(int m) { return (size_t)2 * device_sms() * m * 128 * 4; }

int esp_dense(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats, int n_mats,
              int k2, int cb, void* y, int y_dtype, long long y_stride, void* xh, size_t xh_bytes, float* z,
              size_t z_bytes, int* counters, int n_counters, void* stream) {
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
    DenseParams p = {};
    int nbt = 0;
    RotParams r = {};
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
    p.G = std::min(device_sms(), p.U);
    p.stages = STAGES;
    p.scale = cb_step(cb);
    p.Z = z;
    const size_t zneed = (size_t)2 * p.G * m * 128 * 4;
    ESP_REQUIRE(z && z_bytes >= zneed && aligned(z, 16), ESP_ERR_SCRATCH,
                "esp_dense: Z scratch needs %zu bytes, got %zu", zneed, z_bytes);

    r.x = x;
    r.x_dtype = x_dtype;
    r.x_stride = x_stride;
    r.xh = static_cast<__half*>(xh);
    r.M = m;
    r.Mp = mp;
    r.K = k;
    r.KT = k / 16;
    if (int rc = launch(rot_kernel, dim3((k / 128 + 3) / 4, mp, n_mats), dim3(128), 0, stream, true, r)) return rc;

    int rc = ESP_ERR_UNSUPPORTED;
    switch (cb * 16 + K) {
#define ESP_DENSE_CASE(CB_, K_) \
    case CB_ * 16 + K_: rc = launch_dense_ntg<CB_, K_>(p, stream); break;
        ESP_FOR_EACH_CASE(ESP_DENSE_CASE)
#undef ESP_DENSE_CASE
        default: return set_error(ESP_ERR_UNSUPPORTED, "esp_dense: unsupported codebook/width: cb=%d k2=%d", cb, k2);
    }
    if (rc) return rc;
    return ok();
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
