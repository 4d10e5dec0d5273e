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
 *   z        at least esp_dense_z_bytes(m) bytes, 16-byte aligned (split-K partial sums as tagged 8-byte words),
 *            zero before the first call and left zero by every call that completes (after a call whose device status
 *            is ESP_ERR_TIMEOUT, zero it again)
 *   counters int32, at least sum(n_s)/128 entries, zero (the reference's argument; this kernel does not write it).
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
 * fixed 6.0 MiB array of device memory that every GPU loading the library holds until the process exits.
 * Limits: k <= 4096, sum(n) <= 1,048,576 output columns, m <= 32, a GPU with at most 160 SMs; larger calls return
 * ESP_ERR_INVALID. The first call on a device looks up the array's address (make it before any stream capture).
 * All calls share the array: calls that overlap on the GPU (other streams, other threads) race and must not be made.
 * Results equal esp_dense's. No counterpart in the reference (it has no allocation-free entry point).
 */
int esp_dense_noalloc(const void* x, int x_dtype, long long x_stride, int m, int k, const esp_matrix_t* mats,
                      int n_mats, int k2, int cb, void* y, int y_dtype, long long y_stride, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * MoE routing and grouping. A window is R <= 32 rows with `slots` picks each (k routed, plus the shared expert as
 * the last slot when shared_id >= 0). Grouping: uids[0..ucount) = the distinct expert ids in ascending order, and per
 * distinct expert u its members[u * maxm + j] = row * 32 + slot in (row, slot) order, padded with -1.
 * --------------------------------------------------------------------------------------------------------------- */

/*
 * Router GEMV (x . gate[e] for E experts, plus x . sgate for the shared slot), bf16 rounding of the expert logits,
 * top-k with the lowest id on ties, weights exp(l - l_max) / sum over the k picks, sigmoid of the shared logit, and
 * the grouping, in one launch. Logits are order-fixed fp64 sums of exact products (the CPU oracle reproduces them
 * bit for bit), so the ids equal exact routing's. logits: fp32 [R][E + 1]; counter: int32, zero before the first
 * call and left zero; pick_out / wts_out: [R][k (+1)]. maxm >= R. x / gate / sgate: bf16 or fp16 (x_dtype).
 * Replaces ext().route_group(x, gate, sgate, k, shared_id, logits, counter, pick, wts, uids, ucount, members)
 *                                              (vllm_espalier/csrc/experts.cpp:214-224, route.cu:35-181).
 */
int esp_route_group(const void* x, int x_dtype, long long x_stride, int R, int H, const void* gate, int E,
                    const void* sgate, int k, int shared_id, float* logits, int* counter, int* pick_out, float* wts_out,
                    int* uids, int* ucount, int* members, int maxm, int maxu, void* stream);

/*
 * esp_route_group plus the experts' input rotation in the same launch (this library's fused form, no single counterpart
 * in the reference, which launches rot_in after its routing, experts.py:245-247): once the picks are written, every CTA
 * of the launch computes a share of out0 / out1 [R * slots][H] = fp16(H(x[row] * suh0 / suh1[e]) / sqrt(128)) per
 * 128-block for each slot with a pick e in [0, E_tab), exactly as esp_rot_in. suh0 / suh1: stacked fp16 [E_tab][H].
 * counter: 3 int32 words, zero on entry and left zero.
 */
int esp_route_rot(const void* x, int x_dtype, long long x_stride, int R, int H, const void* gate, int E,
                  const void* sgate, int k, int shared_id, float* logits, int* counter, int* pick_out, float* wts_out,
                  int* uids, int* ucount, int* members, int maxm, int maxu, const uint16_t* suh0,
                  const uint16_t* suh1, uint16_t* out0, uint16_t* out1, int E_tab, void* stream);

/*
 * Grouping of a given pick table pick[R][slots] (ids outside [0, E) are skipped).
 * Replaces ext().group(pick, uids, ucount, members, R, slots, E)  (vllm_espalier/csrc/experts.cpp:79-90,
 *                                                                    experts.cu:23-76).
 */
int esp_group(const int* pick, int R, int slots, int E, int* uids, int* ucount, int* members, int maxm, int maxu,
              void* stream);

/*
 * vLLM's routed picks [R][slots_in] plus the shared expert as an extra last slot with weight sigmoid(x . gate_w)
 * (fp32), written to pick_out / wts_out [R][slots_in + 1], then the grouping.
 * Replaces ext().group_shared(pick_in, wts_in, x, x_stride, gate_w, shared_id, pick_out, wts_out, uids, ucount,
 *                             members, R, slots_in, E)  (vllm_espalier/csrc/experts.cpp:154-173, experts.cu:247-330).
 */
int esp_group_shared(const int* pick_in, const float* wts_in, const void* x, int x_dtype, long long x_stride, int H,
                     const void* gate_w, int shared_id, int* pick_out, float* wts_out, int* uids, int* ucount,
                     int* members, int R, int slots_in, int E, int maxm, int maxu, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Grouped experts. Expert tables are device arrays indexed by expert id: trellis pointers (int64 [E]), half-bits k2
 * (int32 [E]) and kernel codebook ids (int32 [E]); k2_host / cb_host are host copies ([mats][E]) so that the set of
 * (codebook, width) instances is checked on the host. Slot p = row * slots + j; P = rows * slots.
 * --------------------------------------------------------------------------------------------------------------- */

/*
 * out0 / out1 fp16 [P][K] = fp16(H(x[row] * suh0/1[pick[p]]) / sqrt(128)) for every slot with a valid expert.
 * Replaces ext().rot_in(x, x_stride, pick, suh0, suh1, out0, out1, rows, K, slots, E)
 *                                              (vllm_espalier/csrc/experts.cpp:92-104, experts.cu:97-115).
 */
int esp_rot_in(const void* x, int x_dtype, long long x_stride, const int* pick, const uint16_t* suh0,
               const uint16_t* suh1, uint16_t* out0, uint16_t* out1, int rows, int K, int slots, int E, void* stream);

/*
 * Z fp32 [mats][SK][P][N] = the grouped decode GEMV's partial sums of X0/X1 (fp16 [P][K]) against each member's
 * expert matrices, split in SK equal k-slices (the reference's `grouped` contract, its tile parameters nt / warps /
 * pf / lo / hi having no counterpart here).
 * Replaces ext().grouped(X0, X1, TP0, TP1, B0, B1, C0, C1, uids, ucount, members, Z, mats, K, N, P, SK, slots, nt,
 *                        warps, pf, lo, hi)    (vllm_espalier/csrc/experts.cpp:44-66, experts_grouped.cuh).
 */
int esp_grouped(const uint16_t* X0, const uint16_t* X1, const int64_t* TP0, const int64_t* TP1, const int* B0,
                const int* B1, const int* C0, const int* C1, const int* k2_host, const int* cb_host, int E,
                const int* uids, const int* ucount, const int* members, int maxu, int maxm, float* Z, int mats, int K,
                int N, int P, int SK, int slots, void* stream);

/*
 * Fused gate + up + SwiGLU: xd fp16 [P][I] for every slot with a valid expert, equal to grouped(mats = 2) followed
 * by gateup_epilogue(act_mode 1, no limit). S > 1 splits D in S k-slices whose fp32 partials go to Z
 * ([2][S][P][I]) and are added in slice order by the last of the S to finish; counters (int32, maxu * I / 128 + 1,
 * zero and left zero) count the arrivals, the last entry hands out the work items (with counters NULL, allowed when
 * S == 1, items are assigned round robin). No single counterpart: replaces the reference's grouped + gateup_epilogue
 * pair of launches (vllm_espalier/experts.py routed2).
 */
int esp_moe_gateup(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u,
                   const int* k2_g, const int* k2_u, const int* cb_g, const int* cb_u, const int* k2_host,
                   const int* cb_host, int E, const uint16_t* svh_g, const uint16_t* svh_u, const uint16_t* suh_d,
                   const int* uids, const int* ucount, const int* members, int maxu, int maxm, int slots, int P, int D,
                   int I, int S, float* Z, int* counters, uint16_t* xd, void* stream);

/*
 * Fused down + combine: y fp32 [P][D] per slot, out [rows][D] = the routed slots' sum of w * y in slot order (fp32
 * fused multiply-adds from 0) and out_shared [rows][D] = w * y of the shared slot (slot n_routed, when
 * n_routed < slots), both in out_dtype; rows without a valid slot get zeros. counters: int32, rows * D / 128 + 1,
 * zero and left zero (the arrivals, then the work-item counter). Equals grouped(mats = 1) + down_combine2. No single counterpart: replaces the reference's grouped +
 * down_combine2 pair of launches (vllm_espalier/experts.py routed2).
 */
int esp_moe_down(const uint16_t* xd, const int64_t* tp_d, const int* k2_d, const int* cb_d, const int* k2_host,
                 const int* cb_host, int E, const uint16_t* svh_d, const int* uids, const int* ucount,
                 const int* members, int maxu, int maxm, const int* pick, const float* wts, int slots, int n_routed,
                 int rows, int I, int D, float* y, int* counters, void* out, void* out_shared, int out_dtype,
                 void* stream);

/*
 * esp_moe_gateup followed by esp_moe_down in one persistent launch, with the same output bits: gate/up work items are
 * handed out first, a down item starts once its expert's SwiGLU rows are complete (a readiness counter, bounded wait),
 * and a finisher warp does the slice sums, SwiGLU and row combines as their last arrivals land. Tables k2_host /
 * cb_host are [3][E] (gate, up, down). counters: int32, esp_moe_layer_counters(maxu, rows, D, I) entries, zero before
 * the first call and left zero. No single counterpart in the reference (its routed2 runs 4-5 launches for this).
 */
int esp_moe_layer(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u, const int64_t* tp_d,
                  const int* k2_g, const int* k2_u, const int* k2_d, const int* cb_g, const int* cb_u, const int* cb_d,
                  const int* k2_host, const int* cb_host, int E, const uint16_t* svh_g, const uint16_t* svh_u,
                  const uint16_t* suh_d, const uint16_t* svh_d, const int* uids, const int* ucount, const int* members,
                  int maxu, int maxm, const int* pick, const float* wts, int slots, int n_routed, int rows, int D, int I,
                  int S, float* Z, uint16_t* xd, float* y, int* counters, void* out, void* out_shared, int out_dtype,
                  void* stream);
size_t esp_moe_layer_counters(int maxu, int rows, int D, int I);

/*
 * xd fp16 [P][N] from the gate / up partial sums Z [2][SK][P][N] (act_mode 0: bf16-rounded SwiGLU with `limit`,
 * 1: fp32 SwiGLU).
 * Replaces ext().gateup_epilogue(Z, pick, svh_g, svh_u, suh_d, xd, rows, P, N, SK, slots, E, limit, act_mode)
 *                                              (vllm_espalier/csrc/experts.cpp:106-118, experts.cu:120-162).
 */
int esp_gateup_epilogue(const float* Z, const int* pick, const uint16_t* svh_g, const uint16_t* svh_u,
                        const uint16_t* suh_d, uint16_t* xd, int rows, int P, int N, int SK, int slots, int E,
                        float limit, int act_mode, void* stream);

/*
 * y fp32 [P][D] = H(sum of the SK down partials) / sqrt(128) * svh_d; with combine != 0 also out [rows][D] (sum of
 * the first n_routed slots' w * y in slot order) and, when out_shared != NULL, out_shared = w * y of slot n_routed.
 * Replaces ext().down_epilogue (combine = 0), ext().down_combine (fp32 out, n_routed = slots) and
 * ext().down_combine2 (out_dtype out + out_shared)  (vllm_espalier/csrc/experts.cpp:120-129, 139-152, 175-191,
 *                                                     experts.cu:340-393).
 */
int esp_down_combine(const float* Z, const int* pick, const uint16_t* svh_d, float* y, const float* wts, void* out,
                     void* out_shared, int out_dtype, int rows, int P, int D, int SK, int slots, int E, int n_routed,
                     int combine, void* stream);

/*
 * out fp32 [rows][D] = sum over slots of w * y (fused multiply-adds from 0, slot order).
 * Replaces ext().combine(y, wts, out, rows, D, slots)  (vllm_espalier/csrc/experts.cpp:131-137, experts.cu:187-195).
 */
int esp_combine(const float* y, const float* wts, float* out, int rows, int D, int slots, void* stream);

/*
 * Expert-parallel combine on a token's home rank (world ranks; rank q owns routed experts [q E / world,
 * (q + 1) E / world)): out [R][D] = sum over the routed slots j < n_routed, in slot order (fp32 fused multiply-adds
 * from 0), of wts * y, y taken from recv_y fp32 [world][R][slots][D] at the rank owning the slot's expert;
 * out_shared = wts * y of slot n_routed (the shared expert, computed on the home rank) when out_shared != NULL. Same
 * arithmetic as esp_moe_down's combine, so outputs are bit-identical for every world size. No counterpart in the
 * reference (it has no expert parallelism).
 */
int esp_ep_combine(const float* recv_y, const int* pick, const float* wts, void* out, void* out_shared, int out_dtype,
                   int R, int D, int slots, int n_routed, int E_routed, int world, int rank, void* stream);

/*
 * Diagnostic: the bounded wait of the expert kernels on a device flag (int32), on its own. One thread waits until
 * *flag >= need, giving up after 0.2 s (ESP_ERR_TIMEOUT in esp_device_status); *result = 1 if reached, 0 if it gave
 * up. For tests of the timeout path (a flag that nothing sets); no counterpart in the reference.
 */
int esp_wait_flag(const int* flag, int need, int* result, void* stream);

/*
 * Expert-parallel exchange by stores into the other ranks' memory (the ranks of one NVLink box, one process a GPU).
 * No counterpart in the reference (it has no expert parallelism); replaces the two all_to_all collectives of a layer.
 *
 * Set-up, once per rank (not on the decode path): esp_ipc_alloc allocates and zeroes `bytes` of device memory for this
 * rank's inboxes and writes its CUDA IPC handle (esp_ipc_handle_bytes() bytes) to `handle`; the handles are exchanged
 * by the host (any collective) and esp_ipc_open maps another rank's inboxes into this process (no multicast object);
 * esp_ipc_close / esp_ipc_free undo them. Inboxes of a rank: x rows [world][R][D] (x's dtype), picks int32
 * [world][R][slots], y fp32 [R][slots][D], flags_x and flags_y int32 [world]; plus a local epoch word and counters,
 * zero at allocation. Every rank calls with the same R, slots and world; a layer is the routing (esp_route_group of
 * this rank's rows, global ids), then esp_ep_in, the experts, esp_ep_out:
 *
 *   esp_ep_in   x [R][D] (row stride x_stride) and pick [R][slots] (global ids, the shared slot last) of this rank's
 *               rows: each row to the ranks that own one of its routed picks (and to its own rank, which computes its
 *               shared slot), every pick row to every rank (inbox_x / inbox_pick / flags_x: host arrays of every
 *               rank's inbox bases, this rank's own included); then, once every source's flag is seen, local_pick
 *               int32 [world][R][slots] (local expert ids, the local shared entry nl for this rank's own shared
 *               slots, -1 elsewhere), its grouping (uids / ucount / members as esp_group with maxm <= 32), and the
 *               received rows' rotation for the experts (xg / xu [world R slots][D] fp16, as esp_rot_in with the
 *               stacked suh of the local table's nl + 1 entries)
 *   esp_moe_layer_ep  the expert layer over rows = world * R <= 32 received rows (esp_moe_layer's arguments, no
 *               combine): each slot's y row is stored straight into its home rank's inbox_y, and the launch's last
 *               CTA releases every home's flags_y word for this rank; scratch_out: [rows][D] fp32, not read
 *   esp_ep_out  unless `returned` (the rows came from esp_moe_layer_ep), first each locally computed slot's y row
 *               (y fp32 [world][R][slots][D] of esp_moe_layer / esp_moe_down with n_routed = 0) to its home rank's
 *               inbox and the flag (done: int32 [world], zero, left zero); then, once every owner's flag is seen,
 *               out / out_shared [R][D] as esp_ep_combine (slot-ordered fp32 fused multiply-adds; bit-identical to
 *               one GPU); advances *epoch; count: an int32 counter, zero, left zero
 *
 * Waits give up after 0.2 s and record ESP_ERR_TIMEOUT (esp_device_status). The epoch lives on the device, so a
 * CUDA graph of the layer replays correctly.
 */
size_t esp_ipc_handle_bytes(void);
int esp_ipc_alloc(size_t bytes, void** ptr, void* handle);
int esp_ipc_open(const void* handle, void** ptr);
int esp_ipc_close(void* ptr);
int esp_ipc_free(void* ptr);
int esp_ep_in(const void* x, int x_dtype, long long x_stride, int R, int D, const int* pick, int slots, int n_routed,
              int E, int world, int rank, void* const* inbox_x, void* const* inbox_pick, int* const* flags_x,
              const int* epoch, int* local_pick, int* uids, int* ucount, int* members, int maxm, int maxu,
              const void* suh_gate, const void* suh_up, void* xg, void* xu, void* stream);
int esp_moe_layer_ep(const uint16_t* xg, const uint16_t* xu, const int64_t* tp_g, const int64_t* tp_u,
                     const int64_t* tp_d, const int* k2_g, const int* k2_u, const int* k2_d, const int* cb_g,
                     const int* cb_u, const int* cb_d, const int* k2_host, const int* cb_host, int E,
                     const uint16_t* svh_g, const uint16_t* svh_u, const uint16_t* suh_d, const uint16_t* svh_d,
                     const int* uids, const int* ucount, const int* members, int maxu, int maxm,
                     const int* local_pick, const float* no_w, int slots, int rows, int D, int I, int S, float* Z,
                     uint16_t* xd, int* counters, float* const* inbox_y, int* const* flags_y, const int* epoch,
                     int world, int rank, int R, float* scratch_out, void* stream);
int esp_ep_out(const float* y, const int* local_pick, int world, int rank, int R, int slots, int n_routed, int E,
               int D, float* const* inbox_y, int* const* flags_y, const int* pick, const float* wts, void* out,
               void* out_shared, int out_dtype, int* epoch, int* done, int* count, int returned, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ESPALIER_B200_H */
