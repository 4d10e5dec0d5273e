// Expert-parallel MoE exchange over peer memory (one process a GPU, the ranks of one NVLink/NVSwitch box).
//
// Rank q holds routed experts [q E / world, (q + 1) E / world) and the shared expert; each rank routes its own R rows.
// Instead of two collectives a layer, the rows and the results move by stores into the other ranks' memory, mapped
// into this process through CUDA IPC handles (no multicast objects), with release / acquire flags at system scope:
//
//   esp_ep_dispatch  every row to the ranks owning at least one of its routed picks and to its own rank (which
//                    computes the shared slot) (x row: D values), every row's
//                    pick list to every rank; then, per destination, a release store of the call's epoch into that
//                    rank's flag word for this source
//   esp_ep_recv      waits (bounded) for every source's flag, then writes the local pick table: a pick owned here
//                    becomes its local expert id, the shared slot of this rank's own rows the local shared entry, every
//                    other slot -1 (the expert kernels skip it)
//   (grouping, rot_in and the expert kernels run on the received rows, writing y per slot)
//   esp_ep_return    each locally computed slot's y row (D fp32) to its home rank's inbox, then a release flag per
//                    home rank: only owned slots cross NVLink
//   esp_ep_finish    waits (bounded) for every owner's flag, combines each row's routed slots in slot order with fp32
//                    fused multiply-adds from 0 and writes the gated shared slot (the single-GPU layer's arithmetic on
//                    the same y values, so outputs are bit-identical to one GPU), then advances the epoch
//
// The epoch is a device word every kernel of a call reads and the last kernel of the call increments, so a CUDA graph
// of the step replays correctly. A rank writes another rank's inbox for call k + 1 only after its own call k has
// finished, which waited for every owner's return of call k, which each owner issued after reading its own inbox of
// call k: no inbox is overwritten while it is read. Waits give up after WAIT_NS, record ESP_ERR_TIMEOUT and return.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
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

// CTA q: the rows of this rank that have a routed pick owned by rank q (x, D values each; all rows when q is this
// rank, which computes their shared slots) and every row's picks.
__global__ void __launch_bounds__(EP_THREADS) ep_dispatch_kernel(const uint16_t* __restrict__ x, long long x_stride,
                                                                 int R, int D, const int* __restrict__ pick, int slots,
                                                                 int n_routed, int E, int world, int rank,
                                                                 Peers inbox_x, Peers inbox_pick, FlagPeers flags,
                                                                 const int* __restrict__ epoch) {
    pdl_launch_dependents();
    pdl_wait();
    const int q = blockIdx.x;
    uint16_t* dx = static_cast<uint16_t*>(inbox_x.ptr[q]) + (size_t)rank * R * D;
    int* dp = static_cast<int*>(inbox_pick.ptr[q]) + (size_t)rank * R * slots;
    for (int i = threadIdx.x; i < R * slots; i += EP_THREADS) dp[i] = pick[i];
    const int chunks = D / 8;                  // 16-byte pieces of a row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < R; r += EP_THREADS / 32) {
        bool mine = false;
        for (int j = 0; j < n_routed; ++j) {
            const int e = pick[r * slots + j];
            mine |= e >= 0 && e < E && owner_of(e, world, E) == q;
        }
        if (!mine && q != rank) continue;   // the home rank takes all its rows: it computes their shared slots
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)r * x_stride);
        uint4* dst = reinterpret_cast<uint4*>(dx + (size_t)r * D);
        for (int c = lane; c < chunks; c += 32) dst[c] = src[c];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(flags.ptr[q] + rank, *epoch + 1);
    }
}

// One CTA: every source's flag, then the local pick table lp[s][r][j].
__global__ void __launch_bounds__(EP_THREADS) ep_recv_kernel(const int* __restrict__ inbox_pick, const int* flags,
                                                             const int* __restrict__ epoch, int world, int rank, int R,
                                                             int slots, int n_routed, int E, int* __restrict__ lp) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        const int need = *epoch + 1;
        bool ok = true;
        for (int s = 0; s < world && ok; ++s) ok = wait_flag_sys(flags + s, need);
        s_ok = ok;
    }
    __syncthreads();
    const int e0 = rank * E / world, e1 = (rank + 1) * E / world, nl = e1 - e0;
    const int n = world * R * slots;
    for (int i = threadIdx.x; i < n; i += EP_THREADS) {
        int v = -1;
        if (s_ok) {
            const int e = inbox_pick[i];
            const int j = i % slots, s = i / (R * slots);
            if (j < n_routed) v = (e >= e0 && e < e1) ? e - e0 : -1;
            else v = (s == rank && e >= 0) ? nl : -1;   // the shared slot: computed on the row's home rank only
        }
        lp[i] = v;
    }
}

// CTA h (grid x = world): this rank's y rows of the slots whose home is rank h, into h's inbox [R][slots][D], then a
// release flag in h's flag word for this owner. Other CTAs along y share the copying of one home's rows.
__global__ void __launch_bounds__(EP_THREADS) ep_return_kernel(const float* __restrict__ y, const int* __restrict__ lp,
                                                               int R, int slots, int D, int rank, Peers inbox_y,
                                                               FlagPeers flags, const int* __restrict__ epoch,
                                                               int* __restrict__ done) {
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpc = EP_THREADS / 32, nw = wpc * gridDim.y;
    float* dst = static_cast<float*>(inbox_y.ptr[h]);
    const int base = h * R * slots;
    for (int i = blockIdx.y * wpc + warp; i < R * slots; i += nw) {
        if (lp[base + i] < 0) continue;
        const float4* src = reinterpret_cast<const float4*>(y + (size_t)(base + i) * D);
        float4* d = reinterpret_cast<float4*>(dst + (size_t)i * D);
        for (int c = lane; c < D / 4; c += 32) d[c] = src[c];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();   // this CTA's stores before the arrival that may release the flag
        if (atomicAdd(done + h, 1) == (int)gridDim.y - 1) {
            __threadfence_system();
            done[h] = 0;
            st_release_sys(flags.ptr[h] + rank, *epoch + 1);
        }
    }
}

// One CTA a row: every owner's flag, then out[r] = slot-ordered fp32 fma of the routed slots' y from 0, and
// out_shared[r] = w_shared * y_shared (esp_ep_combine's arithmetic); the last CTA advances the epoch.
template <typename T>
__global__ void __launch_bounds__(EP_THREADS) ep_finish_kernel(const float* __restrict__ inbox_y, const int* flags,
                                                               const int* __restrict__ pick, const float* __restrict__ wts,
                                                               T* __restrict__ out, T* __restrict__ out_shared, int R,
                                                               int D, int slots, int n_routed, int E, int world,
                                                               int* epoch, int* count) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ int s_ok;
    const int r = blockIdx.x;
    if (threadIdx.x == 0) {
        const int need = *epoch + 1;
        bool ok = true;
        for (int s = 0; s < world && ok; ++s) ok = wait_flag_sys(flags + s, need);
        s_ok = ok;
    }
    __syncthreads();
    if (s_ok) {
        for (int n = threadIdx.x; n < D; n += EP_THREADS) {
            float acc = 0.f;
            for (int j = 0; j < n_routed; ++j) {
                const int e = pick[r * slots + j];
                if (e < 0 || e >= E) continue;
                acc = __fmaf_rn(wts[r * slots + j], inbox_y[((size_t)r * slots + j) * D + n], acc);
            }
            out[(size_t)r * D + n] = from_f32<T>(acc);
            if (out_shared && slots > n_routed) {
                const int j = n_routed;
                const float v = pick[r * slots + j] >= 0 ? wts[r * slots + j] * inbox_y[((size_t)r * slots + j) * D + n]
                                                         : 0.f;
                out_shared[(size_t)r * D + n] = from_f32<T>(v);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(count, 1) == (int)gridDim.x - 1) {
        *count = 0;
        *epoch += 1;
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

int esp_ep_dispatch(const void* x, int x_dtype, long long x_stride, int R, int D, const int* pick, int slots,
                    int n_routed, int E, int world, int rank, void* const* inbox_x, void* const* inbox_pick,
                    int* const* flags_x, const int* epoch, void* stream) {
    ESP_REQUIRE(x && pick && inbox_x && inbox_pick && flags_x && epoch, ESP_ERR_INVALID, "ep_dispatch: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world, ESP_ERR_INVALID,
                "ep_dispatch: 1 to %d ranks", EP_MAX_WORLD);
    ESP_REQUIRE(x_dtype == ESP_DTYPE_BF16 || x_dtype == ESP_DTYPE_F16, ESP_ERR_INVALID, "ep_dispatch: bf16/fp16 rows");
    ESP_REQUIRE(R >= 1 && R <= 32 && D % 8 == 0 && x_stride >= D && x_stride % 8 == 0 && aligned(x, 16),
                ESP_ERR_INVALID, "ep_dispatch: 1..32 rows of 16-byte aligned D values");
    ESP_REQUIRE(slots >= 1 && slots <= 32 && n_routed <= slots && E >= world, ESP_ERR_INVALID, "ep_dispatch: slots");
    Peers px = {}, pp = {};
    FlagPeers pf = {};
    for (int q = 0; q < world; ++q) {
        ESP_REQUIRE(inbox_x[q] && inbox_pick[q] && flags_x[q], ESP_ERR_INVALID, "ep_dispatch: rank %d's buffers", q);
        px.ptr[q] = inbox_x[q];
        pp.ptr[q] = inbox_pick[q];
        pf.ptr[q] = flags_x[q];
    }
    if (int rc = launch(ep_dispatch_kernel, dim3(world), dim3(EP_THREADS), 0, stream, true,
                        static_cast<const uint16_t*>(x), x_stride, R, D, pick, slots, n_routed, E, world, rank, px, pp,
                        pf, epoch))
        return rc;
    return ok();
}

int esp_ep_recv(const int* inbox_pick, const int* flags_x, const int* epoch, int world, int rank, int R, int slots,
                int n_routed, int E, int* local_pick, void* stream) {
    ESP_REQUIRE(inbox_pick && flags_x && epoch && local_pick, ESP_ERR_INVALID, "ep_recv: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world && R >= 1 && R <= 32 &&
                    slots >= 1 && slots <= 32 && n_routed <= slots && E >= world,
                ESP_ERR_INVALID, "ep_recv: limits");
    if (int rc = launch(ep_recv_kernel, dim3(1), dim3(EP_THREADS), 0, stream, true, inbox_pick, flags_x, epoch, world,
                        rank, R, slots, n_routed, E, local_pick))
        return rc;
    return ok();
}

int esp_ep_return(const float* y, const int* local_pick, int world, int rank, int R, int slots, int D,
                  float* const* inbox_y, int* const* flags_y, const int* epoch, int* done, void* stream) {
    ESP_REQUIRE(y && local_pick && inbox_y && flags_y && epoch && done, ESP_ERR_INVALID, "ep_return: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world && R >= 1 && R <= 32 &&
                    slots >= 1 && slots <= 32 && D % 4 == 0,
                ESP_ERR_INVALID, "ep_return: limits");
    Peers py = {};
    FlagPeers pf = {};
    for (int q = 0; q < world; ++q) {
        ESP_REQUIRE(inbox_y[q] && flags_y[q], ESP_ERR_INVALID, "ep_return: rank %d's buffers", q);
        py.ptr[q] = inbox_y[q];
        pf.ptr[q] = flags_y[q];
    }
    const int split = R * slots > 64 ? 4 : 1;
    if (int rc = launch(ep_return_kernel, dim3(world, split), dim3(EP_THREADS), 0, stream, true, y, local_pick, R,
                        slots, D, rank, py, pf, epoch, done))
        return rc;
    return ok();
}

int esp_ep_finish(const float* inbox_y, const int* flags_y, const int* pick, const float* wts, void* out,
                  void* out_shared, int out_dtype, int R, int D, int slots, int n_routed, int E, int world, int* epoch,
                  int* count, void* stream) {
    ESP_REQUIRE(inbox_y && flags_y && pick && wts && out && epoch && count, ESP_ERR_INVALID, "ep_finish: null pointer");
    ESP_REQUIRE(world >= 1 && world <= EP_MAX_WORLD && R >= 1 && R <= 32 && slots >= 1 && slots <= 32 &&
                    n_routed <= slots && E >= world,
                ESP_ERR_INVALID, "ep_finish: limits");
    ESP_REQUIRE(out_dtype == ESP_DTYPE_BF16 || out_dtype == ESP_DTYPE_F16 || out_dtype == ESP_DTYPE_F32, ESP_ERR_INVALID,
                "ep_finish: dtype");
    int rc;
    if (out_dtype == ESP_DTYPE_BF16)
        rc = launch(ep_finish_kernel<__nv_bfloat16>, dim3(R), dim3(EP_THREADS), 0, stream, true, inbox_y, flags_y, pick,
                    wts, static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(out_shared), R, D, slots,
                    n_routed, E, world, epoch, count);
    else if (out_dtype == ESP_DTYPE_F16)
        rc = launch(ep_finish_kernel<__half>, dim3(R), dim3(EP_THREADS), 0, stream, true, inbox_y, flags_y, pick, wts,
                    static_cast<__half*>(out), static_cast<__half*>(out_shared), R, D, slots, n_routed, E, world, epoch,
                    count);
    else
        rc = launch(ep_finish_kernel<float>, dim3(R), dim3(EP_THREADS), 0, stream, true, inbox_y, flags_y, pick, wts,
                    static_cast<float*>(out), static_cast<float*>(out_shared), R, D, slots, n_routed, E, world, epoch,
                    count);
    if (rc) return rc;
    return ok();
}

}  // extern "C"
