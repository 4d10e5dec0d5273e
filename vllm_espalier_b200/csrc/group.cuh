// Device helpers shared by the routing and the expert-parallel kernels: the grouping of a pick table (distinct
// experts in id order, members in (row, slot) order), GPU-scope release / acquire flags with bounded waits, and the
// experts' input rotation of a share of the picked slots (rot_in's arithmetic).
#pragma once

#include "common.cuh"

namespace esp {
namespace {

constexpr int MAX_E = 512;              // experts (incl. the shared slot) the grouping handles
constexpr int MAX_PICKS = 8 * 32 * 9;   // rows x slots of one window (8 ranks x 32 rows x 9 slots on an EP receiver)

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

// Distinct experts (< n_ids) of picks[0..n) in id order -> uids / ucount; per expert its members i (row * 32 + slot,
// i = row * slots + slot) in order, padded with -1 to maxm. An expert with more than maxm members takes
// ceil(count / maxm) consecutive entries (the same id, members in order, maxm an entry): never the case for a window
// of at most maxm rows, where every expert has at most one member a row. One CTA; picks in shared memory.
__device__ void group_block(const int* sh_pick, int n, int slots, int n_ids, int* __restrict__ uids,
                            int* __restrict__ ucount, int* __restrict__ members, int maxm, int maxu) {
    __shared__ int warp_tot[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int per = (n_ids + blockDim.x - 1) / blockDim.x;    // ids a thread (<= 2 with 256 threads, 512 ids)
    int cnt[2] = {0, 0};
    int used = 0;                                             // entries of this thread's ids
    for (int q = 0; q < per && q < 2; ++q) {
        const int e = threadIdx.x * per + q;
        int c = 0;
        if (e < n_ids)
            for (int i = 0; i < n; ++i) c += sh_pick[i] == e;
        cnt[q] = c;
        used += (c + maxm - 1) / maxm;
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
    for (int q = 0; q < per && q < 2; ++q) {
        if (cnt[q] == 0) continue;
        const int e = threadIdx.x * per + q;
        int j = 0;                                            // member index within the current entry
        for (int i = 0; i < n; ++i)
            if (sh_pick[i] == e) {
                if (j == maxm) {                              // entry full: the next entry of the same id
                    ++place;
                    j = 0;
                }
                if (place < maxu) {
                    if (j == 0) uids[place] = e;
                    members[place * maxm + j] = (i / slots) * 32 + (i % slots);
                }
                ++j;
            }
        if (place < maxu)
            for (; j < maxm; ++j) members[place * maxm + j] = -1;
        ++place;
    }
}


// The experts' input rotation folded into the routing launch (esp_route_rot): once the last CTA has written the picks,
// every CTA of the launch (one wave, all resident) rotates a share of the (matrix, slot, 128-block) items:
// out_m[p] = fp16(H(x[row] * suh_m[e]) / sqrt(128)), rot_in's arithmetic, for each slot p with a pick e in [0, E_tab).
struct RotIn {
    const __half* suh[2];          // stacked [E_tab][H] (gate, up); null: no rotation
    __half* out[2];                // [R * slots][H]
    int E_tab;
};

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// one thread: wait until *flag >= need (GPU-scope acquire), bounded by time
__device__ bool wait_flag_gpu(const int* flag, int need) {
    if (ld_acquire_gpu(flag) >= need) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        for (int i = 0; i < 32; ++i) {
            __nanosleep(32);
            if (ld_acquire_gpu(flag) >= need) return true;
        }
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS) break;
        if (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT) return false;
    }
    report(ESP_ERR_TIMEOUT);
    return false;
}

// The rotation of the items (matrix, slot p, 128-block) with a pick in [0, E_tab): pick_of(p) gives slot p's entry.
template <typename T, typename PickOf>
__device__ void rotate_share_by(const T* __restrict__ x, long long x_stride, int H, int P, int slots, const RotIn& rot,
                                PickOf pick_of) {
    const int lane = threadIdx.x & 31;
    const int nblk = H / 128, ntask = 2 * P * nblk;
    const int wpc = blockDim.x >> 5, nw = gridDim.x * gridDim.y * wpc;
    for (int w = (blockIdx.y * gridDim.x + blockIdx.x) * wpc + (threadIdx.x >> 5); w < ntask; w += nw) {
        const int mat = w / (P * nblk), rem = w % (P * nblk), p = rem / nblk, blk = rem % nblk;
        const int e = pick_of(p);
        if (e < 0 || e >= rot.E_tab) continue;
        const int k0 = blk * 128 + 4 * lane;
        const __half* su = rot.suh[mat] + (size_t)e * H + k0;
        const T* xr = x + (size_t)(p / slots) * x_stride + k0;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __fmul_rn(to_f<T>(xr[j]), __half2float(su[j]));
        fwht128(v, lane);
        const __half2 a = __floats2half2_rn(v[0] * HAD_SCALE, v[1] * HAD_SCALE);
        const __half2 b = __floats2half2_rn(v[2] * HAD_SCALE, v[3] * HAD_SCALE);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&a);
        u.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(rot.out[mat] + (size_t)p * H + k0) = u;
    }
}

template <typename T>
__device__ void rotate_share(const T* __restrict__ x, long long x_stride, int H, const int* pick, int P, int slots,
                             const RotIn& rot) {
    rotate_share_by<T>(x, x_stride, H, P, slots, rot, [pick](int p) { return __ldcg(pick + p); });
}

}  // namespace
}  // namespace esp
