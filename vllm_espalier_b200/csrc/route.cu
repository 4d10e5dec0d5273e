// MoE routing: router GEMV + softmax / top-k / renormalisation + the shared-expert gate + grouping in one launch, and
// the grouping kernels the reference exposes separately (group, group_shared).
//
// Reference behaviour (vllm_espalier/csrc/route.cu:35-181, experts.cu:23-76, 247-330): logits of the E experts are
// rounded to bf16 and top-k is taken with the lowest expert id winning ties; the k weights are renormalised to sum 1;
// the shared slot (id shared_id) gets sigmoid(x . sgate) in fp32; grouping lists the distinct experts in id order and,
// per expert, its members row * 32 + slot in (row, slot) order, padded with -1.
//
// Exactness (expert ids bit-exact against exact routing): each logit is an order-fixed fp64 reduction of the exact
// bf16 x bf16 products (lane l of a warp keeps 8 partial sums s_q of the products j = 8 l + 256 i + q, i ascending;
// the lane's value is ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)); the 32 lane values meet in an xor tree
// over offsets 16..1), rounded once to bf16. The CPU oracle (oracle/espalier_oracle.c orc_router_logit) is the same
// order, so ids match bit for bit, and the fp64 sum is exact to far below bf16 resolution, so they equal the
// correctly rounded logits' choice. Top-k compares bf16 logit values (exp is monotone), so the choice does not depend
// on the exponential's last bit.
//
// B200 layout: a warp a logit column (E experts + the shared gate), one wave of CTAs (one an SM) over a 2-D grid of
// column groups x row-pair groups, each CTA looping over its row pairs with all of a pair's loads in flight at once;
// the last CTA to arrive (acq_rel counter) stages the logits in shared memory, does the per-row selection (a warp a
// row) and the grouping (members written in parallel over the picks), then resets the counter.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "group.cuh"
#include "host.hpp"

ESP_DEFINE_STATUS_READER(route)

namespace esp {
namespace {

constexpr int RT = 256;                 // threads a CTA
constexpr int RW = RT / 32;
constexpr int MAX_K = 16;


// fp64 logits of up to RB rows against one weight row, each in the documented order: lane l keeps 8 partial sums s_q,
// adding the product x[j] * w[j] (formed in fp32, exact for bf16 / fp16 pairs unless below 2^-126, then widened) for
// j = 8 l + 256 i + q, i ascending; the lane's value is ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)); the lanes
// meet in an xor tree over offsets 16..1. Every lane returns the full sums. The 8 * RB chains are independent; all of
// the lane's loads are issued before the first addition (H <= 2048: at most 8 chunks of 8 a lane).
constexpr int RB = 2;   // rows a warp

template <typename T>
__device__ __forceinline__ void add_chunk(const uint4& a4, const float (&wf)[8], double (&s)[8]) {
    const T* a = reinterpret_cast<const T*>(&a4);
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] = __dadd_rn(s[q], (double)__fmul_rn(to_f<T>(a[q]), wf[q]));
}

constexpr int MAXC = 8;   // 8-value chunks a lane keeps in registers (H <= 2048)

// The lane's chunks of a weight row: loaded before the kernel waits for the previous one (weights are not its output).
template <typename T>
__device__ __forceinline__ void load_w(const T* __restrict__ w, int H, int lane, uint4 (&uw)[MAXC]) {
    const int nc = (H - 8 * lane + 255) / 256;
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
        if (i < nc) uw[i] = *reinterpret_cast<const uint4*>(w + 8 * lane + 256 * i);
}

template <typename T>
__device__ __forceinline__ void logits64(const T* __restrict__ x, long long x_stride, int nr, const T* __restrict__ w,
                                         const uint4 (&uw)[MAXC], int H, int lane, double (&acc)[RB]) {
    uint4 ux[RB][MAXC];
    const int nc = (H - 8 * lane + 255) / 256;
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
        if (i < nc) {
#pragma unroll
            for (int r = 0; r < RB; ++r)
                if (r < nr) ux[r][i] = *reinterpret_cast<const uint4*>(x + (size_t)r * x_stride + 8 * lane + 256 * i);
        }
    double s[RB][8];
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int q = 0; q < 8; ++q) s[r][q] = 0.0;
#pragma unroll
    for (int i = 0; i < MAXC; ++i)
        if (i < nc) {
            float wf[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) wf[q] = to_f<T>(reinterpret_cast<const T*>(&uw[i])[q]);
#pragma unroll
            for (int r = 0; r < RB; ++r)
                if (r < nr) add_chunk<T>(ux[r][i], wf, s[r]);
        }
    for (int j0 = 8 * lane + 256 * MAXC; j0 < H; j0 += 256) {     // longer rows
        const uint4 b4 = *reinterpret_cast<const uint4*>(w + j0);
        float wf[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) wf[q] = to_f<T>(reinterpret_cast<const T*>(&b4)[q]);
#pragma unroll
        for (int r = 0; r < RB; ++r)
            if (r < nr) add_chunk<T>(*reinterpret_cast<const uint4*>(x + (size_t)r * x_stride + j0), wf, s[r]);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        acc[r] = __dadd_rn(__dadd_rn(__dadd_rn(s[r][0], s[r][1]), __dadd_rn(s[r][2], s[r][3])),
                           __dadd_rn(__dadd_rn(s[r][4], s[r][5]), __dadd_rn(s[r][6], s[r][7])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r] = __dadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
    }
}

// Top-k keys: a bf16 logit and its id as one 32-bit key whose unsigned order is (value, then lower id) order: the
// value's bits mapped to an order-preserving 16-bit code (-0 taken as +0, as a float compare does), then 0xffff - id.
__device__ __forceinline__ uint32_t topk_key(float v, int e) {
    const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
    const uint32_t k16 = (b & 0x80000000u) ? (~b >> 16) : ((b >> 16) | 0x8000u);
    return (k16 << 16) | (0xffffu - (uint32_t)e);
}
__device__ __forceinline__ float topk_value(uint32_t key) {
    const uint32_t k16 = key >> 16;
    const uint32_t b16 = (k16 & 0x8000u) ? (k16 ^ 0x8000u) : (~k16 & 0xffffu);
    return __uint_as_float(b16 << 16);
}

__device__ __forceinline__ float round_bf16_d(double v) {
    // round the fp64 value once to bf16 (nearest even), via the exact fp64 -> bf16 conversion
    return __bfloat162float(__double2bfloat16(v));
}

// The grouping of route's own picks, whose ids are distinct within a row (top-k of distinct ids plus the shared id)
// and whose rows number at most 32: a row bitmask an id (shared-memory atomicOr), the distinct ids in id order by a
// block scan, then an id's members row by row (ascending) with the slot found in that row. Same output as group_block.
__device__ void group_distinct(const int* sh_pick, int R, int slots, int n_ids, int* __restrict__ uids,
                               int* __restrict__ ucount, int* __restrict__ members, int maxm, int maxu) {
    __shared__ unsigned sh_mask[MAX_E];
    __shared__ int sh_place[MAX_E];
    __shared__ int warp_tot[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = threadIdx.x; e < n_ids; e += blockDim.x) sh_mask[e] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < R * slots; i += blockDim.x) {
        const int e = sh_pick[i];
        if (e >= 0 && e < n_ids) atomicOr(&sh_mask[e], 1u << (i / slots));
    }
    __syncthreads();
    const int per = (n_ids + blockDim.x - 1) / blockDim.x;    // ids a thread (<= 2 with 256 threads, 512 ids)
    unsigned mk[2] = {0u, 0u};
    int used = 0;
    for (int q = 0; q < per && q < 2; ++q) {
        const int e = threadIdx.x * per + q;
        mk[q] = e < n_ids ? sh_mask[e] : 0u;
        used += mk[q] != 0u;
    }
    int inc = used;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int v = lane < nw ? warp_tot[lane] : 0;
        int s = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x2 = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += x2;
        }
        if (lane < nw) warp_tot[lane] = s - v;
        if (lane == 31) ucount[0] = s;
    }
    __syncthreads();
    int place = warp_tot[warp] + inc - used;
    for (int q = 0; q < per && q < 2; ++q) {   // an id's entry: its id and the padding after its members
        const unsigned m = mk[q];
        if (m == 0u) continue;
        const int e = threadIdx.x * per + q;
        sh_place[e] = place;
        if (place < maxu) {
            uids[place] = e;
            for (int j = __popc(m); j < maxm; ++j) members[place * maxm + j] = -1;
        }
        ++place;
    }
    __syncthreads();
    // the members, one pick a thread: a pick of row r is its id's member number popc(rows of the id before r)
    for (int i = threadIdx.x; i < R * slots; i += blockDim.x) {
        const int e = sh_pick[i];
        if (e < 0 || e >= n_ids) continue;
        const int r = i / slots;
        const int j = __popc(sh_mask[e] & ((1u << r) - 1u));
        const int at = sh_place[e];
        if (at < maxu && j < maxm) members[at * maxm + j] = r * 32 + (i - r * slots);
    }
}

template <typename T>
__global__ void __launch_bounds__(RT) route_kernel(const T* __restrict__ x, long long x_stride, int R, int H,
                                                   const T* __restrict__ gate, int E, const T* __restrict__ sgate,
                                                   int k, int shared_id, float* __restrict__ logits,
                                                   int* __restrict__ counter, int* __restrict__ pick_out,
                                                   float* __restrict__ wts_out, int* __restrict__ uids,
                                                   int* __restrict__ ucount, int* __restrict__ members, int maxm,
                                                   int maxu, int rpc, const RotIn rot) {
    __shared__ int last;
    __shared__ int sh_pick[MAX_PICKS];
    extern __shared__ float sh_logit[];    // [R][C], the last CTA's copy of the logits
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int has = shared_id >= 0;
    const int C = E + has;                 // logit columns: experts, then the shared gate
    const int slots = k + has;
    const int c = blockIdx.x * RW + warp;      // a warp a logit column, rpc rows a CTA, RB at a time
    const int r0 = blockIdx.y * rpc;
    const T* w = c < E ? gate + (size_t)c * H : sgate;
    uint4 uw[MAXC];
    if (c < C) load_w<T>(w, H, lane, uw);      // the router's weights overlap the previous kernel's tail
    pdl_wait();
    if (c < C)
        for (int rb = r0; rb < min(R, r0 + rpc); rb += RB) {
            const int nr = min(RB, R - rb);
            double acc[RB];
            logits64<T>(x + (size_t)rb * x_stride, x_stride, nr, w, uw, H, lane, acc);
#pragma unroll
            for (int r = 0; r < RB; ++r)
                if (r < nr && lane == 0) logits[(size_t)(rb + r) * C + c] = c < E ? round_bf16_d(acc[r]) : (float)acc[r];
        }
    __syncthreads();
    if (threadIdx.x == 0) {
        last = arrive_acq_rel(counter) == (int)(gridDim.x * gridDim.y) - 1;
    }
    __syncthreads();
    const int ncta = gridDim.x * gridDim.y;
    if (!last) {
        if (!rot.suh[0]) return;
        // the rotation share of this CTA once the last CTA has published the picks (counter[1]); counter[2] counts
        // the CTAs done, the last of which clears both words for the next call
        __shared__ int ok;
        if (threadIdx.x == 0) ok = wait_flag_gpu(counter + 1, 1);
        __syncthreads();
        if (ok) rotate_share<T>(x, x_stride, H, pick_out, R * (k + (shared_id >= 0)), k + (shared_id >= 0), rot);
        __syncthreads();
        if (threadIdx.x == 0 && arrive_acq_rel(counter + 2) == ncta - 1) {
            counter[1] = 0;
            counter[2] = 0;
        }
        return;
    }
    for (int i = threadIdx.x; i < R * C; i += RT) sh_logit[i] = __ldcg(logits + i);   // one round of loads
    __syncthreads();

    // per row (a warp a row): top-k of the bf16 logits, lowest id on ties (a warp max over the keys a pick, the
    // winner's key cleared); lane t keeps pick t; weights exp(l_t - l_0) / sum, summed in pick order
    for (int r = warp; r < R; r += RW) {
        const float* lr = sh_logit + (size_t)r * C;
        uint32_t key[MAX_E / 32];
#pragma unroll
        for (int q = 0; q < MAX_E / 32; ++q) {
            const int e = lane + 32 * q;
            key[q] = e < E ? topk_key(lr[e], e) : 0u;
        }
        int my_id = 0;
        float my_v = 0.f;
        for (int t = 0; t < k; ++t) {
            uint32_t m = key[0];
#pragma unroll
            for (int q = 1; q < MAX_E / 32; ++q) m = max(m, key[q]);
            const uint32_t best = __reduce_max_sync(0xffffffffu, m);
#pragma unroll
            for (int q = 0; q < MAX_E / 32; ++q)
                if (key[q] == best) key[q] = 0u;
            if (lane == t) {
                my_id = (int)(0xffffu - (best & 0xffffu));
                my_v = topk_value(best);
            }
        }
        const float v0 = __shfl_sync(0xffffffffu, my_v, 0);
        const float pt = expf(my_v - v0);
        float sum = 0.f;
        for (int t = 0; t < k; ++t) sum += __shfl_sync(0xffffffffu, pt, t);
        if (lane < k) {
            pick_out[r * slots + lane] = my_id;
            sh_pick[r * slots + lane] = my_id;
            wts_out[r * slots + lane] = pt / sum;
        }
        if (has && lane == 0) {
            pick_out[r * slots + k] = shared_id;
            sh_pick[r * slots + k] = shared_id;
            wts_out[r * slots + k] = 1.f / (1.f + expf(-lr[E]));
        }
    }
    __syncthreads();   // the picks are in sh_pick (written beside pick_out above)
    if (rot.suh[0]) {   // publish the picks to the other CTAs first: their rotation overlaps the grouping
        if (threadIdx.x == 0) {
            __threadfence();
            st_release_gpu(counter + 1, 1);
        }
    }
    group_distinct(sh_pick, R, slots, E + has, uids, ucount, members, maxm, maxu);
    if (threadIdx.x == 0) *counter = 0;
    if (rot.suh[0]) {
        rotate_share<T>(x, x_stride, H, pick_out, R * slots, slots, rot);
        __syncthreads();
        if (threadIdx.x == 0 && arrive_acq_rel(counter + 2) == ncta - 1) {
            counter[1] = 0;
            counter[2] = 0;
        }
    }
}

// group (experts.cu:23-76): the grouping of a given pick table.
__global__ void __launch_bounds__(RT) group_kernel(const int* __restrict__ pick, int n, int slots, int E,
                                                   int* __restrict__ uids, int* __restrict__ ucount,
                                                   int* __restrict__ members, int maxm, int maxu) {
    __shared__ int sh_pick[MAX_PICKS];
    pdl_launch_dependents();
    pdl_wait();
    for (int i = threadIdx.x; i < n; i += RT) sh_pick[i] = pick[i];
    __syncthreads();
    group_block(sh_pick, n, slots, E, uids, ucount, members, maxm, maxu);
}

// group_shared (experts.cu:247-330): routed picks plus the shared slot (weight sigmoid(x . gate_w), fp32 in a fixed
// per-thread order then a fixed tree), then the grouping.
template <typename T>
__global__ void __launch_bounds__(RT) group_shared_kernel(const int* __restrict__ pick_in, const float* __restrict__ wts_in,
                                                          const T* __restrict__ x, long long x_stride,
                                                          const T* __restrict__ gate_w, int H, int shared_id,
                                                          int* __restrict__ pick_out, float* __restrict__ wts_out,
                                                          int* __restrict__ uids, int* __restrict__ ucount,
                                                          int* __restrict__ members, int R, int slots_in, int E,
                                                          int maxm, int maxu) {
    __shared__ int sh_pick[MAX_PICKS];
    __shared__ float red[RW];
    pdl_launch_dependents();
    pdl_wait();
    const int has = shared_id >= 0;
    const int slots = slots_in + has;
    const int n = R * slots;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < n; i += RT) {
        const int r = i / slots, q = i % slots;
        const int e = q < slots_in ? pick_in[r * slots_in + q] : shared_id;
        sh_pick[i] = e;
        pick_out[i] = e;
        if (q < slots_in) wts_out[i] = wts_in[r * slots_in + q];
    }
    if (has) {
        for (int r = 0; r < R; ++r) {
            float acc = 0.f;
            for (int j = threadIdx.x; j < H; j += RT) acc = fmaf(to_f<T>(x[(size_t)r * x_stride + j]), to_f<T>(gate_w[j]), acc);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) red[warp] = acc;
            __syncthreads();
            if (warp == 0) {
                float v = lane < RW ? red[lane] : 0.f;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) wts_out[r * slots + slots_in] = 1.f / (1.f + expf(-v));
            }
            __syncthreads();
        }
    }
    __syncthreads();
    group_block(sh_pick, n, slots, E, uids, ucount, members, maxm, maxu);
}

int route_launch(const void* x, int x_dtype, long long x_stride, int R, int H, const void* gate, int E,
                 const void* sgate, int k, int shared_id, float* logits, int* counter, int* pick_out, float* wts_out,
                 int* uids, int* ucount, int* members, int maxm, int maxu, const RotIn& rot, void* stream) {
    ESP_REQUIRE(x && gate && logits && counter && pick_out && wts_out && uids && ucount && members, ESP_ERR_INVALID,
                "route_group: null pointer");
    const int has = shared_id >= 0;
    ESP_REQUIRE(x_dtype == ESP_DTYPE_BF16 || x_dtype == ESP_DTYPE_F16, ESP_ERR_INVALID, "route_group: x must be bf16 or fp16");
    ESP_REQUIRE(E >= 1 && E + has <= MAX_E && k >= 1 && k <= MAX_K && k <= E && H % 256 == 0 && H > 0, ESP_ERR_INVALID,
                "route_group: shape limits");
    ESP_REQUIRE(R >= 1 && R <= 32 && k + has <= 32, ESP_ERR_INVALID, "route_group: at most 32 rows and 32 slots");
    ESP_REQUIRE(!has || sgate, ESP_ERR_INVALID, "the shared gate weight is needed with a shared slot");
    ESP_REQUIRE(aligned(x, 16) && aligned(gate, 16) && (!has || aligned(sgate, 16)) && x_stride % 8 == 0,
                ESP_ERR_INVALID, "route_group: rows must be 16-byte aligned");
    ESP_REQUIRE(maxm >= R && maxu >= 1, ESP_ERR_INVALID, "route_group: members must hold R entries an expert");
    const int C = E + has;
    // one wave: a CTA an SM (the kernel's registers allow one), the row pairs spread over what the columns leave
    const int gx = (C + RW - 1) / RW, pairs = (R + RB - 1) / RB;
    const int ry = std::max(1, std::min(pairs, device_sms() / gx));
    const int ppc = (pairs + ry - 1) / ry;    // row pairs a CTA
    const dim3 grid((unsigned)gx, (unsigned)((pairs + ppc - 1) / ppc));
    const size_t smem = (size_t)R * C * sizeof(float);
    static bool opted[2] = {false, false};
    const int ti = x_dtype == ESP_DTYPE_BF16 ? 0 : 1;
    if (!opted[ti]) {
        const int rc0 = ti == 0 ? allow_smem(route_kernel<__nv_bfloat16>, (size_t)32 * MAX_E * sizeof(float))
                                : allow_smem(route_kernel<__half>, (size_t)32 * MAX_E * sizeof(float));
        if (rc0) return rc0;
        opted[ti] = true;
    }
    int rc;
    if (x_dtype == ESP_DTYPE_BF16)
        rc = launch(route_kernel<__nv_bfloat16>, grid, dim3(RT), smem, stream, true,
                    static_cast<const __nv_bfloat16*>(x), x_stride, R, H, static_cast<const __nv_bfloat16*>(gate), E,
                    static_cast<const __nv_bfloat16*>(sgate), k, shared_id, logits, counter, pick_out, wts_out, uids,
                    ucount, members, maxm, maxu, ppc * RB, rot);
    else
        rc = launch(route_kernel<__half>, grid, dim3(RT), smem, stream, true, static_cast<const __half*>(x), x_stride,
                    R, H, static_cast<const __half*>(gate), E, static_cast<const __half*>(sgate), k, shared_id, logits,
                    counter, pick_out, wts_out, uids, ucount, members, maxm, maxu, ppc * RB, rot);
    if (rc) return rc;
    return ok();
}

}  // namespace
}  // namespace esp

using namespace esp;

extern "C" {

int esp_route_group(const void* x, int x_dtype, long long x_stride, int R, int H, const void* gate, int E,
                    const void* sgate, int k, int shared_id, float* logits, int* counter, int* pick_out, float* wts_out,
                    int* uids, int* ucount, int* members, int maxm, int maxu, void* stream) {
    return route_launch(x, x_dtype, x_stride, R, H, gate, E, sgate, k, shared_id, logits, counter, pick_out, wts_out,
                        uids, ucount, members, maxm, maxu, RotIn{}, stream);
}

int esp_route_rot(const void* x, int x_dtype, long long x_stride, int R, int H, const void* gate, int E,
                  const void* sgate, int k, int shared_id, float* logits, int* counter, int* pick_out, float* wts_out,
                  int* uids, int* ucount, int* members, int maxm, int maxu, const uint16_t* suh0,
                  const uint16_t* suh1, uint16_t* out0, uint16_t* out1, int E_tab, void* stream) {
    ESP_REQUIRE(suh0 && suh1 && out0 && out1 && E_tab >= 1, ESP_ERR_INVALID, "route_rot: rotation buffers");
    ESP_REQUIRE(H % 128 == 0 && aligned(suh0, 8) && aligned(suh1, 8) && aligned(out0, 8) && aligned(out1, 8),
                ESP_ERR_INVALID, "route_rot: 8-byte aligned rotation buffers");
    RotIn rot = {};
    rot.suh[0] = reinterpret_cast<const __half*>(suh0);
    rot.suh[1] = reinterpret_cast<const __half*>(suh1);
    rot.out[0] = reinterpret_cast<__half*>(out0);
    rot.out[1] = reinterpret_cast<__half*>(out1);
    rot.E_tab = E_tab;
    return route_launch(x, x_dtype, x_stride, R, H, gate, E, sgate, k, shared_id, logits, counter, pick_out, wts_out,
                        uids, ucount, members, maxm, maxu, rot, stream);
}

int esp_group(const int* pick, int R, int slots, int E, int* uids, int* ucount, int* members, int maxm, int maxu,
              void* stream) {
    ESP_REQUIRE(pick && uids && ucount && members, ESP_ERR_INVALID, "group: null pointer");
    ESP_REQUIRE(E >= 1 && E <= MAX_E, ESP_ERR_INVALID, "too many experts for the grouping kernel");
    ESP_REQUIRE(slots >= 1 && slots <= 32, ESP_ERR_INVALID, "at most 32 slots a row");
    ESP_REQUIRE(R >= 1 && R * slots <= MAX_PICKS, ESP_ERR_INVALID, "grouping window too large");
    ESP_REQUIRE(maxm >= 1 && maxu >= 1, ESP_ERR_INVALID, "members too small");
    if (int rc = launch(group_kernel, dim3(1), dim3(RT), 0, stream, true, pick, R * slots, slots, E, uids, ucount,
                        members, maxm, maxu))
        return rc;
    return ok();
}

int esp_group_shared(const int* pick_in, const float* wts_in, const void* x, int x_dtype, long long x_stride, int H,
                     const void* gate_w, int shared_id, int* pick_out, float* wts_out, int* uids, int* ucount,
                     int* members, int R, int slots_in, int E, int maxm, int maxu, void* stream) {
    ESP_REQUIRE(pick_in && wts_in && x && pick_out && wts_out && uids && ucount && members, ESP_ERR_INVALID,
                "group_shared: null pointer");
    ESP_REQUIRE(E >= 1 && E <= MAX_E, ESP_ERR_INVALID, "too many experts for the grouping kernel");
    const int slots = slots_in + (shared_id >= 0);
    ESP_REQUIRE(slots <= 32 && R >= 1 && R * slots <= MAX_PICKS, ESP_ERR_INVALID, "grouping window too large");
    ESP_REQUIRE(shared_id < 0 || gate_w, ESP_ERR_INVALID, "a shared slot needs its gate weight");
    ESP_REQUIRE(x_dtype == ESP_DTYPE_BF16 || x_dtype == ESP_DTYPE_F16, ESP_ERR_INVALID, "x: bf16/fp16");
    int rc;
    if (x_dtype == ESP_DTYPE_BF16)
        rc = launch(group_shared_kernel<__nv_bfloat16>, dim3(1), dim3(RT), 0, stream, true, pick_in, wts_in,
                    static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(gate_w), H,
                    shared_id, pick_out, wts_out, uids, ucount, members, R, slots_in, E, maxm, maxu);
    else
        rc = launch(group_shared_kernel<__half>, dim3(1), dim3(RT), 0, stream, true, pick_in, wts_in,
                    static_cast<const __half*>(x), x_stride, static_cast<const __half*>(gate_w), H, shared_id, pick_out,
                    wts_out, uids, ucount, members, R, slots_in, E, maxm, maxu);
    if (rc) return rc;
    return ok();
}

}  // extern "C"
