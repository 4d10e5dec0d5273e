// Expert-parallel MoE exchange over peer memory (one process a GPU, the ranks of one NVLink/NVSwitch box).
//
// Rank q holds routed experts [q E / world, (q + 1) E / world) and the shared expert; each rank routes its own R rows.
// Instead of two collectives a layer, the rows and the results move by stores into the other ranks' memory, mapped
// into this process through CUDA IPC handles (no multicast objects), with release / acquire flags at system scope.
// A layer is four launches: routing, esp_ep_in, the expert layer kernel, esp_ep_out.
//
//   esp_ep_in   (dispatch) CTA q < world stores every row of this rank that has a routed pick owned by rank q (all
//               rows when q is this rank, which computes their shared slots) and every row's pick list into rank q's
//               inboxes, then a release store of the call's epoch into q's flag word for this source;
//               (receive) every CTA waits (bounded) for every source's flag; CTA 0 writes the local pick table (a pick
//               owned here becomes its local expert id, the shared slot of this rank's own rows the local shared
//               entry, every other slot -1) and its grouping (esp_group's); every CTA rotates a share of the received
//               slots' rows for the expert kernel (rot_in), mapping each slot's pick to its local entry itself
//   the expert kernel (esp_moe_layer_ep, moe.cu) stores each slot's y row into its home rank's inbox and releases the
//               flags; above 32 received rows the two-launch expert kernels write y locally and esp_ep_out returns it
//   esp_ep_out  (return, only then) CTAs (h, part) store each locally computed slot's y row (D fp32) into home rank
//               h's inbox, then a release flag per home rank: only owned slots cross NVLink;
//               (finish) CTA r waits (bounded) for every owner's flag and combines row r's routed slots in slot order
//               with fp32 fused multiply-adds from 0 and the gated shared slot (the single-GPU layer's arithmetic on
//               the same y values, so outputs are bit-identical to one GPU); the last CTA advances the epoch
//
// The epoch is a device word every kernel of a call reads and the last CTA of esp_ep_out increments once every CTA
// of that launch has read it, so a CUDA graph of the step replays correctly. A rank writes another rank's inbox for
// call k + 1 only after its own call k has finished, which waited for every owner's return of call k, which each
// owner issued after reading its own inbox of call k: no inbox is overwritten while it is read. Waits give up after
// WAIT_NS, record ESP_ERR_TIMEOUT and return.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "group.cuh"
#include "host.hpp"

ESP_DEFINE_STATUS_READER(ep)

namespace esp {
namespace {

constexpr int EP_MAX_WORLD = 8;
constexpr int EP_THREADS = 256;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// one thread: wait until *flag >= need (system-scope acquire), bounded by WAIT_NS
__device__ bool wait_flag_sys(const int* flag, int need) {
    if (ld_acquire_sys(flag) >= need) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        for (int i = 0; i < 32; ++i) {
            __nanosleep(32);
            if (ld_acquire_sys(flag) >= need) return true;
        }
        const uint64_t dt = global_ns() - t0;
        if (dt > WAIT_NS) break;
        if (dt > 20000 && *reinterpret_cast<volatile int*>(&g_device_status) == ESP_ERR_TIMEOUT) return false;
    }
    report(ESP_ERR_TIMEOUT);
    return false;
}

struct Peers {
    void* ptr[EP_MAX_WORLD];
};
struct FlagPeers {
    int* ptr[EP_MAX_WORLD];
};

__device__ __forceinline__ int owner_of(int e, int world, int E) { return ((e + 1) * world - 1) / E; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }

struct InParams {
    const uint16_t* x;                 // this rank's rows [R] (row stride x_stride), bf16 / fp16 bits
    long long x_stride;
    int R, D, slots, n_routed, E, world, rank;
    const int* pick;                   // this rank's picks [R][slots], global ids (the shared slot last, id E)
    Peers inbox_x, inbox_pick;         // every rank's inboxes: x [world][R][D], picks [world][R][slots]
    FlagPeers flags_x;                 // every rank's flag words [world] (one a source)
    const int* epoch;
    const int* my_pick;                // this rank's inboxes and flags
    const int* my_flags;
    int* lp;                           // out: local pick table [world][R][slots]
    int* uids; int* ucount; int* members;
    int maxm, maxu;
    RotIn rot;                         // suh (stacked [nl + 1][D], gate / up) and the rotated rows [world R slots][D]
};

// Dispatch, receive, group and rotate in one launch (see the top of the file). x of dtype T.
template <typename T>
__global__ void __launch_bounds__(EP_THREADS) ep_in_kernel(const __grid_constant__ InParams p) {
    __shared__ int sh_lp[MAX_PICKS];
    __shared__ int s_ok;
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = p.R, D = p.D, slots = p.slots;
    if ((int)blockIdx.x < p.world) {   // ---- dispatch to rank q ----
        const int q = blockIdx.x;
        uint16_t* dx = static_cast<uint16_t*>(p.inbox_x.ptr[q]) + (size_t)p.rank * R * D;
        int* dp = static_cast<int*>(p.inbox_pick.ptr[q]) + (size_t)p.rank * R * slots;
        for (int i = threadIdx.x; i < R * slots; i += EP_THREADS) dp[i] = p.pick[i];
        for (int r = warp; r < R; r += EP_THREADS / 32) {
            bool mine = false;
            for (int j = 0; j < p.n_routed; ++j) {
                const int e = p.pick[r * slots + j];
                mine |= e >= 0 && e < p.E && owner_of(e, p.world, p.E) == q;
            }
            if (!mine && q != p.rank) continue;   // the home rank takes all its rows: it computes their shared slots
            const uint4* src = reinterpret_cast<const uint4*>(p.x + (size_t)r * p.x_stride);
            uint4* dst = reinterpret_cast<uint4*>(dx + (size_t)r * D);
            for (int c = lane; c < D / 8; c += 32) dst[c] = src[c];
        }
        __syncthreads();
        // the release is cumulative over the CTA's stores ordered before it by the barrier: no separate fence
        if (threadIdx.x == 0) st_release_sys(p.flags_x.ptr[q] + p.rank, *p.epoch + 1);
    }
    const int e0 = p.rank * p.E / p.world, e1 = (p.rank + 1) * p.E / p.world, nl = e1 - e0;
    const int n = p.world * R * slots;
    // ---- receive: every CTA waits for every source's flag itself (no publication step inside the launch) ----
    if (threadIdx.x == 0) {
        const int need = *p.epoch + 1;
        bool ok = true;
        for (int s = 0; s < p.world && ok; ++s) ok = wait_flag_sys(p.my_flags + s, need);
        s_ok = ok;
    }
    __syncthreads();
    // slot i's local entry: a routed pick owned here -> its local id, this rank's own shared slot -> nl, else -1
    auto local_of = [&](int i) -> int {
        if (!s_ok) return -1;
        const int e = __ldcv(p.my_pick + i);
        const int j = i % slots, src = i / (R * slots);
        if (j < p.n_routed) return (e >= e0 && e < e1) ? e - e0 : -1;
        return (src == p.rank && e >= 0) ? nl : -1;
    };
    if (blockIdx.x == 0) {             // the local table and its grouping, for the expert kernel
        for (int i = threadIdx.x; i < n; i += EP_THREADS) {
            const int v = local_of(i);
            sh_lp[i] = v;
            p.lp[i] = v;
        }
        __syncthreads();
        group_block(sh_lp, n, slots, nl + 1, p.uids, p.ucount, p.members, p.maxm, p.maxu);
    }
    // ---- rotate a share of the received slots (rot_in's arithmetic), each slot's entry from the picks directly ----
    rotate_share_by<T>(reinterpret_cast<const T*>(p.inbox_x.ptr[p.rank]), D, D, n, slots, p.rot, local_of);
}

struct OutParams {
    const float* y;                    // this rank's expert output [world][R][slots][D] fp32
    const int* lp;                     // the local pick table of the call
    int R, D, slots, n_routed, E, world, rank, split;
    Peers inbox_y;                     // every rank's inbox [R][slots][D] fp32
    FlagPeers flags_y;
    const int* my_flags;
    const float* my_y;                 // this rank's inbox
    const int* pick;                   // this rank's picks [R][slots] (global ids) and weights
    const float* wts;
    void* out; void* out_shared;       // [R][D] of dtype T
    int* epoch;
    int* done;                         // [world], zero on entry and left zero
    int* count;                        // zero on entry and left zero
};

// Return and finish in one launch (see the top of the file): CTAs [0, world * split) return, CTA world * split + r
// finishes row r. Every CTA is resident (at most 8 * 4 + 32), so the finishing CTAs' waits on this rank's own
// returns end.
template <typename T>
__global__ void __launch_bounds__(EP_THREADS) ep_out_kernel(const __grid_constant__ OutParams p) {
    __shared__ int s_ok;
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = p.R, D = p.D, slots = p.slots;
    const int need = *p.epoch + 1;
    const int nret = p.world * p.split;   // 0: the expert kernel stored the y rows and released the flags itself
    if ((int)blockIdx.x < nret) {      // ---- return: this rank's y rows of home h's slots ----
        const int h = blockIdx.x / p.split, part = blockIdx.x % p.split;
        const int wpc = EP_THREADS / 32, nw = wpc * p.split;
        float* dst = static_cast<float*>(p.inbox_y.ptr[h]);
        const int base = h * R * slots;
        for (int i = part * wpc + warp; i < R * slots; i += nw) {
            if (__ldcg(p.lp + base + i) < 0) continue;
            const float4* src = reinterpret_cast<const float4*>(p.y + (size_t)(base + i) * D);
            float4* d = reinterpret_cast<float4*>(dst + (size_t)i * D);
            for (int c = lane; c < D / 4; c += 32) d[c] = __ldcg(src + c);
        }
        __syncthreads();
        // the arrival releases this CTA's stores (cumulative over the barrier), the last one acquires the others'
        // and its system-scope release of the flag publishes them all: no separate fences
        if (threadIdx.x == 0 && arrive_acq_rel(p.done + h) == p.split - 1) {
            p.done[h] = 0;
            st_release_sys(p.flags_y.ptr[h] + p.rank, need);
        }
    } else {                           // ---- finish row r ----
        const int r = blockIdx.x - nret;
        if (threadIdx.x == 0) {
            bool ok = true;
            for (int s = 0; s < p.world && ok; ++s) ok = wait_flag_sys(p.my_flags + s, need);
            s_ok = ok;
        }
        __syncthreads();
        if (s_ok) {
            // four columns a thread at a time, eight slots' loads in flight before their fused multiply-adds (the
            // same per-element order as one slot after the other: slot order from 0, picks outside [0, E) skipped)
            T* out = static_cast<T*>(p.out);
            T* out_shared = static_cast<T*>(p.out_shared);
            const float* yr = p.my_y + (size_t)r * slots * D;
            const int* pk = p.pick + r * slots;
            const float* wt = p.wts + r * slots;
            for (int c = 4 * threadIdx.x; c < D; c += 4 * EP_THREADS) {
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                for (int j0 = 0; j0 < p.n_routed; j0 += 8) {
                    float4 v[8];
                    bool on[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int j = j0 + q;
                        on[q] = j < p.n_routed && pk[j] >= 0 && pk[j] < p.E;
                        if (on[q]) v[q] = __ldcv(reinterpret_cast<const float4*>(yr + (size_t)j * D + c));
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        if (on[q]) {
                            const float w = wt[j0 + q];
                            acc[0] = __fmaf_rn(w, v[q].x, acc[0]);
                            acc[1] = __fmaf_rn(w, v[q].y, acc[1]);
                            acc[2] = __fmaf_rn(w, v[q].z, acc[2]);
                            acc[3] = __fmaf_rn(w, v[q].w, acc[3]);
                        }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) out[(size_t)r * D + c + i] = from_f32<T>(acc[i]);
                if (out_shared && slots > p.n_routed) {
                    const int j = p.n_routed;
                    float sh[4] = {0.f, 0.f, 0.f, 0.f};
                    if (pk[j] >= 0) {
                        const float4 y4 = __ldcv(reinterpret_cast<const float4*>(yr + (size_t)j * D + c));
                        const float w = wt[j];
                        sh[0] = w * y4.x; sh[1] = w * y4.y; sh[2] = w * y4.z; sh[3] = w * y4.w;
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) out_shared[(size_t)r * D + c + i] = from_f32<T>(sh[i]);
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(p.count, 1) == (int)gridDim.x - 1) {   // every CTA has read the epoch
        *p.count = 0;
        *p.epoch += 1;
    }
}

}  // namespace
}  // namespace esp

using namespace esp;

extern "C" {

size_t esp_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int esp_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    ESP_REQUIRE(ptr && handle && bytes > 0, ESP_ERR_INVALID, "esp_ipc_alloc: arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    ESP_REQUIRE(e == cudaSuccess, ESP_ERR_CUDA, "esp_ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return set_error(ESP_ERR_CUDA, "esp_ipc_alloc: %s", cudaGetErrorString(e));
    }
    *ptr = p;
    return ok();
}

int esp_ipc_open(const void* handle, void** ptr) {
    ESP_REQUIRE(handle && ptr, ESP_ERR_INVALID, "esp_ipc_open: arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    ESP_REQUIRE(e == cudaSuccess, ESP_ERR_CUDA, "esp_ipc_open: %s", cudaGetErrorString(e));
    return ok();
}

int esp_ipc_close(void* ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    ESP_REQUIRE(e == cudaSuccess, ESP_ERR_CUDA, "esp_ipc_close: %s", cudaGetErrorString(e));
    return ok();
}

int esp_ipc_free(void* ptr) {
    const cudaError_t e = cudaFree(ptr);
    ESP_REQUIRE(e == cudaSuccess, ESP_ERR_CUDA, "esp_ipc_free: %s", cudaGetErrorString(e));
    return ok();
}

int esp_ep_in(const void* x, int x_dtype, long long x_stride, int R, int D, const int* pick, int slots, int n_routed,
              int E, int world, int rank, void* const* inbox_x, void* const* inbox_pick, int* const* flags_x,
              const int* epoch, int* local_pick, int* uids, int* ucount, int* members, int maxm, int maxu,
              const void* suh_gate, const void* suh_up, void* xg, void* xu, void* stream) {
    ESP_REQUIRE(x && pick && inbox_x && inbox_pick && flags_x && epoch && local_pick && uids && ucount && members &&
                    suh_gate && suh_up && xg && xu,
                ESP_ERR_INVALID, "ep_in: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world, ESP_ERR_INVALID,
                "ep_in: 1 to %d ranks", EP_MAX_WORLD);
    ESP_REQUIRE(x_dtype == ESP_DTYPE_BF16 || x_dtype == ESP_DTYPE_F16, ESP_ERR_INVALID, "ep_in: bf16/fp16 rows");
    ESP_REQUIRE(R >= 1 && R <= 32 && D % 128 == 0 && x_stride >= D && x_stride % 8 == 0 && aligned(x, 16),
                ESP_ERR_INVALID, "ep_in: 1..32 rows of 16-byte aligned D values (D a multiple of 128)");
    ESP_REQUIRE(slots >= 1 && slots <= 32 && n_routed <= slots && E >= world && world * R * slots <= MAX_PICKS,
                ESP_ERR_INVALID, "ep_in: slots");
    const int nl = (rank + 1) * E / world - rank * E / world;
    ESP_REQUIRE(nl + 1 <= MAX_E && maxm >= 1 && maxm <= 32 && maxu >= 1, ESP_ERR_INVALID, "ep_in: grouping limits");
    InParams p{};
    p.x = static_cast<const uint16_t*>(x);
    p.x_stride = x_stride;
    p.R = R; p.D = D; p.slots = slots; p.n_routed = n_routed; p.E = E; p.world = world; p.rank = rank;
    p.pick = pick;
    for (int q = 0; q < world; ++q) {
        ESP_REQUIRE(inbox_x[q] && inbox_pick[q] && flags_x[q], ESP_ERR_INVALID, "ep_in: rank %d's buffers", q);
        p.inbox_x.ptr[q] = inbox_x[q];
        p.inbox_pick.ptr[q] = inbox_pick[q];
        p.flags_x.ptr[q] = flags_x[q];
    }
    p.epoch = epoch;
    p.my_pick = static_cast<const int*>(inbox_pick[rank]);
    p.my_flags = flags_x[rank];
    p.lp = local_pick;
    p.uids = uids; p.ucount = ucount; p.members = members; p.maxm = maxm; p.maxu = maxu;
    p.rot.suh[0] = static_cast<const __half*>(suh_gate);
    p.rot.suh[1] = static_cast<const __half*>(suh_up);
    p.rot.out[0] = static_cast<__half*>(xg);
    p.rot.out[1] = static_cast<__half*>(xu);
    p.rot.E_tab = nl + 1;
    // about four rotation tasks (a matrix, a slot, a 128-block) a warp, at least a CTA a destination, one wave
    const int tasks = 2 * world * R * slots * (D / 128);
    const int grid = std::max(world, std::min(device_sms(), (tasks + 4 * (EP_THREADS / 32) - 1) / (4 * (EP_THREADS / 32))));
    int rc = x_dtype == ESP_DTYPE_BF16
                 ? launch(ep_in_kernel<__nv_bfloat16>, dim3(grid), dim3(EP_THREADS), 0, stream, true, p)
                 : launch(ep_in_kernel<__half>, dim3(grid), dim3(EP_THREADS), 0, stream, true, p);
    if (rc) return rc;
    return ok();
}

int esp_ep_out(const float* y, const int* local_pick, int world, int rank, int R, int slots, int n_routed, int E,
               int D, float* const* inbox_y, int* const* flags_y, const int* pick, const float* wts, void* out,
               void* out_shared, int out_dtype, int* epoch, int* done, int* count, int returned, void* stream) {
    ESP_REQUIRE(inbox_y && flags_y && pick && wts && out && epoch && count && (returned || (y && local_pick && done)),
                ESP_ERR_INVALID, "ep_out: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world && R >= 1 && R <= 32 &&
                    slots >= 1 && slots <= 32 && n_routed <= slots && E >= world && D % 4 == 0,
                ESP_ERR_INVALID, "ep_out: limits");
    ESP_REQUIRE(out_dtype == ESP_DTYPE_BF16 || out_dtype == ESP_DTYPE_F16 || out_dtype == ESP_DTYPE_F32, ESP_ERR_INVALID,
                "ep_out: dtype");
    OutParams p{};
    p.y = y; p.lp = local_pick;
    p.R = R; p.D = D; p.slots = slots; p.n_routed = n_routed; p.E = E; p.world = world; p.rank = rank;
    p.split = returned ? 0 : R * slots > 64 ? 4 : 1;
    for (int q = 0; q < world; ++q) {
        ESP_REQUIRE(inbox_y[q] && flags_y[q], ESP_ERR_INVALID, "ep_out: rank %d's buffers", q);
        p.inbox_y.ptr[q] = inbox_y[q];
        p.flags_y.ptr[q] = flags_y[q];
    }
    p.my_flags = flags_y[rank];
    p.my_y = inbox_y[rank];
    p.pick = pick; p.wts = wts; p.out = out; p.out_shared = out_shared;
    p.epoch = epoch; p.done = done; p.count = count;
    const dim3 grid(world * p.split + R);
    int rc;
    if (out_dtype == ESP_DTYPE_BF16) rc = launch(ep_out_kernel<__nv_bfloat16>, grid, dim3(EP_THREADS), 0, stream, true, p);
    else if (out_dtype == ESP_DTYPE_F16) rc = launch(ep_out_kernel<__half>, grid, dim3(EP_THREADS), 0, stream, true, p);
    else rc = launch(ep_out_kernel<float>, grid, dim3(EP_THREADS), 0, stream, true, p);
    if (rc) return rc;
    return ok();
}

}  // extern "C"
