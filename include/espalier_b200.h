/*
 * espalier_b200 — C ABI of the B200-native Espalier decode hot path.
 *
 * One shared library (libespalier_b200.so) with plain-pointer entry points: no torch or C++ types cross this
 * boundary. Every entry point validates its arguments on the host, enqueues its kernels on the given CUDA stream
 * (a cudaStream_t passed as void*, NULL = the legacy default stream) and returns ESP_OK or an error code; the message
 * of the last error on the calling thread is available from esp_last_error(). Nothing here allocates device memory,
 * synchronises the stream, or traps on the device: scratch buffers are the caller's, and device-side bounded waits
 * that give up record ESP_ERR_TIMEOUT, read with esp_device_status().
 *
 * Each entry point names the reference binding it replaces (the reference plugin geodesa-ai/vllm-espalier, its
 * pybind module vllm_espalier/csrc/experts.cpp, reached through vllm_espalier/experts.py ext()).
 *
 * fp16 / bf16 data are passed as uint16_t bit patterns. Trellises are the checkpoint's int16
 * [in/16][out/16][16*K] tensors, read in place.
 */
#ifndef ESPALIER_B200_H
#define ESPALIER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define ESP_OK 0
#define ESP_ERR_INVALID 1     /* bad shape, pointer, alignment or argument */
#define ESP_ERR_UNSUPPORTED 2 /* no kernel for this (codebook, width) */
#define ESP_ERR_SCRATCH 3     /* a caller-provided scratch buffer is too small */
#define ESP_ERR_CUDA 4        /* a CUDA runtime call or launch failed */
#define ESP_ERR_TIMEOUT 5     /* a bounded device-side wait gave up (read by esp_device_status) */

/* element types of activations / outputs */
#define ESP_DTYPE_F16 0
#define ESP_DTYPE_BF16 1
#define ESP_DTYPE_F32 2

/* kernel codebook ids (the reference's KERNEL_CB values, vllm_espalier/experts.py:34) */
#define ESP_CB_MCG 1
#define ESP_CB_E2M1 3
#define ESP_CB_INT5 6
#define ESP_CB_INT6 7

/* Library version (major * 10000 + minor * 100 + patch). */
int esp_version(void);

/* Message of the last error returned on this thread ("" after success). */
const char* esp_last_error(void);

/* Device-side status word of the current device (ESP_OK or ESP_ERR_TIMEOUT); reset != 0 clears it. Synchronous. */
int esp_device_status(int* status, int reset);

/* Number of streaming multiprocessors of the current device (cached). */
int esp_sm_count(void);

/*
 * W fp16 [kin][n] = decoded weights of one trellis, bit-identical to the reference's decode.
 * Replaces ext().dequant(T, out, k2, cb)      (vllm_espalier/csrc/experts.cpp:68-77, experts_grouped.cuh:321-340).
 */
int esp_dequant(const int16_t* trellis, int kin, int n, int k2, int cb, uint16_t* out, void* stream);

/*
 * y fp16 [m][k] = fp16(H(x * pre) / sqrt(128) * post) along rows of 128; pre / post may be NULL; y may alias x.
 * Replaces ext().had(x, pre, post, y)         (vllm_espalier/csrc/experts.cpp:226-232, dense.cu:242-265).
 */
int esp_had(const uint16_t* x, int m, int k, const uint16_t* pre, const uint16_t* post, uint16_t* y, void* stream);

/* One Espalier matrix of a dense layer. */
typedef struct esp_matrix {
    const int16_t* trellis; /* [k/16][n/16][8*k2] */
    const uint16_t* suh;    /* fp16 [k] input signs */
    const uint16_t* svh;    /* fp16 [n] output scales */
    int n;                  /* output features, a multiple of 128 */
    int col0;               /* first column of this matrix in y */
} esp_matrix_t;

/*
 * Dense layer decode (1..32 rows): y[:, col0_s : col0_s + n_s] = H(H(x * suh_s) @ W_s) * svh_s for up to 4 matrices
 * sharing k, codebook and width, in two launches (input rotation, then the fused decode GEMV with its output
 * rotation). x: [m][k] of x_dtype with row stride x_stride elements; y: [m][*] of y_dtype, row stride y_stride.
 * Scratch (caller-owned, never resized here):
 *   xh       fp16, at least esp_dense_xh_bytes(m, k, n_mats) bytes (rotated activations)
 *   z        fp32, at least esp_dense_z_bytes(m) bytes (split-K partial sums)
 *   counters int32, at least sum(n_s)/128 entries, zero before the first call and left zero by every call.
 * Results are row-invariant (a row's bits never depend on the other rows) and deterministic.
 * Replaces ext().dense(x, T[], suh[], svh[], col0[], y, xh, Z, counters, k2, cb, SK, W, PF, rot_smem)
 *                                              (vllm_espalier/csrc/experts.cpp:193-211, dense.cu:276-340).
 */
int esp_dense(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats, int n_mats,
              int k2, int cb, void* y, int y_dtype, long long y_stride, void* xh, size_t xh_bytes, float* z,
              size_t z_bytes, int* counters, int n_counters, void* stream);
size_t esp_dense_xh_bytes(int m, int k, int n_mats);
size_t esp_dense_z_bytes(int m);

/*
 * esp_dense without any scratch argument and without allocating: for callers that cannot allocate device memory when
 * they run a layer (a serving engine whose KV cache already holds nearly all of HBM, a host bound only through this
 * C ABI with no allocator, a path that must not take cudaMalloc's implicit synchronisation). The scratch lives in one
 * fixed 3.6 MiB array of device memory that every GPU loading the library holds until the process exits.
 * Limits: k <= 4096, sum(n) <= 1,048,576 output columns, m <= 32, a GPU with at most 160 SMs; larger calls return
 * ESP_ERR_INVALID. The first call on a device looks up the array's address (make it before any stream capture).
 * All calls share the array: calls that overlap on the GPU (other streams, other threads) race and must not be made.
 * Results equal esp_dense's. No counterpart in the reference (it has no allocation-free entry point).
 */
int esp_dense_noalloc(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats,
                      int n_mats, int k2, int cb, void* y, int y_dtype, long long y_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ESPALIER_B200_H */
