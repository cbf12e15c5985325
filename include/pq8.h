/*
 * pq8 - B200 (sm_100a) Q8_0-weight x FP32-activation contraction library.
 *
 * C ABI: plain pointers and sizes, no exceptions or aborts cross it. Every
 * function returns 0 on success or an error code: values below 1000 are
 * CUDA runtime error numbers, values from 1000 up are PQ8_ERR_* below.
 * pq8_error_string() names any code.
 *
 * Pointers marked "device" are device addresses in the current CUDA context
 * of the calling thread (the primary context, as the reference's ctypes
 * driver uses it). `stream` is a cudaStream_t / CUstream; NULL is the legacy
 * default stream, which is what the reference launches on. Work is enqueued
 * asynchronously on that stream; the library never synchronizes except in
 * pq8_device_status(). It never allocates device memory: scratch space is a
 * caller-provided workspace, in the manner of cublasSetWorkspace_v2.
 *
 * Weights are kept resident in the "packed Q8_0" device format produced by
 * pq8_pack_q8_0*() from GGUF Q8_0 blocks (34-byte `<f2 scale><32 x i8>`
 * records along K, row-major [N, K]): a 256-byte header, then per tile of
 * 128 weight rows and per 32-wide K block a 4352-byte record holding the
 * int8 values (16-byte aligned, laid out for coalesced and tensor-memory
 * access) followed by the 128 fp16 scales. The packed format is what makes
 * the GGUF blocks, whose 34-byte stride breaks 16-byte TMA alignment,
 * streamable by bulk copies.
 *
 * Reference interfaces replaced (mgostIH/parakeet_cuda):
 *   - parakeet_cuda/gpu.py:169-184  GPU.load_weights -> dequant_q8 expansion
 *   - parakeet_cuda/gpu.py:87-90    Blas.linear -> cublasSgemm_v2 (FP32)
 *   - parakeet_cuda/kernels/runtime.cu:26-33   dequant_q8
 *   - parakeet_cuda/kernels/runtime.cu:180-188 q8_gemv
 *   - parakeet_cuda/kernels/runtime.cu:49-62   silu / residual / bias_act / glu epilogues
 *   - parakeet_cuda/kernels/runtime.cu:155-179 lstm / joint_relu / argmax_tdt
 *   - kernels/q8_gemm.cu:5-42                  q8_gemm (direct fused-dequant GEMM)
 */
#ifndef PQ8_H
#define PQ8_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PQ8_API __attribute__((visibility("default")))
#else
#define PQ8_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes (>= 1000; smaller nonzero values are cudaError_t) ---- */
#define PQ8_OK 0
#define PQ8_ERR_INVALID_ARGUMENT 1001  /* NULL pointer, negative size, bad enum */
#define PQ8_ERR_UNSUPPORTED_SHAPE 1002 /* K not a positive multiple of 32, N out of range, ... */
#define PQ8_ERR_MISALIGNED 1003        /* a pointer does not meet the documented alignment */
#define PQ8_ERR_ARCH 1004              /* current device is not compute capability 10.0 (sm_100a) */
#define PQ8_ERR_WORKSPACE 1005         /* workspace NULL or smaller than pq8_*_workspace_size() */
#define PQ8_ERR_LAYOUT 1006            /* device-side: packed header does not match n/k/layout */
#define PQ8_ERR_TIMEOUT 1007           /* device-side: a bounded wait inside a kernel expired */
#define PQ8_ERR_DRIVER 1008            /* CUDA driver entry point missing or tensor-map encode failed */
#define PQ8_ERR_LIBRARY 1009           /* a cuBLAS call of pq8_rel_attention failed */

/* ---- packed weight layouts ---- */
#define PQ8_LAYOUT_ROWS 0   /* packed row p = source row p */
#define PQ8_LAYOUT_GLU 1    /* rows j and j+N/2 paired in one warp; output width N/2 */
#define PQ8_LAYOUT_GATES4 2 /* LSTM gates i,f,g,o of one hidden unit in one tile column; output width N/4 */

/* ---- epilogues (applied to z = acc + bias; bias may be NULL) ---- */
#define PQ8_EPI_NONE 0     /* y = z                              (Blas.linear, + bias_act relu=0) */
#define PQ8_EPI_RELU 1     /* y = max(z, 0)                      (bias_act relu=1) */
#define PQ8_EPI_SILU 2     /* y = z * sigmoid(z)                 (FFN linear1 + silu) */
#define PQ8_EPI_GLU 3      /* y[:, j] = z[:, j] * sigmoid(z[:, j+N/2])   (pointwise_conv1 + glu; GLU layout) */
#define PQ8_EPI_RESIDUAL 4 /* y = resid + alpha * z              (linear + residual; y may alias resid) */

/* ---- flags ---- */
#define PQ8_FLAG_X_TF32 1   /* x already holds TF32-rounded values: skip the in-kernel rounding pass */
#define PQ8_FLAG_OUT_TF32 2 /* round y to TF32 (nearest) so that it can feed another GEMM with PQ8_FLAG_X_TF32 */
#define PQ8_FLAG_FP32_PRODUCTS 4 /* pq8_rel_attention, pq8_stem: cuBLAS products in FP32 instead of TF32 */
#define PQ8_ATTN_FP32 PQ8_FLAG_FP32_PRODUCTS

#define PQ8_HEADER_BYTES 256
#define PQ8_TILE_ROWS 128
#define PQ8_RECORD_BYTES 4352 /* 128 rows x 32 int8 + 128 fp16 scales */
#define PQ8_GEMV_MAX_M 64        /* the GEMV entry points (pq8_gemv, pq8_lstm_layer, pq8_joint_argmax) take m <= 64 */
#define PQ8_LINEAR_GEMV_MAX_M 8  /* pq8_linear sends m <= 8 to pq8_gemv; 9..64 to whichever kernel a
                                    measured cost model finds faster for (m, n, k); larger m to pq8_gemm */

/* Name of an error code (static string; never NULL). */
PQ8_API const char* pq8_error_string(int code);

/* Library version as major*10000 + minor*100 + patch. */
PQ8_API int pq8_version(void);

/* ---- host-side packing (no GPU needed) ---------------------------------
 * Replaces the per-layer upload + dequant_q8 expansion of GPU.load_weights
 * (parakeet_cuda/gpu.py:169-184): the Q8_0 bytes stay Q8_0, only their order
 * changes, and the result is uploaded once and kept resident.
 */

/* Bytes of a packed tensor of n rows x k columns in `layout`. */
PQ8_API int pq8_packed_size(int n, int k, int layout, size_t* bytes);

/* Pack GGUF Q8_0 blocks (host memory, n*k/32 records of 34 bytes, row-major
 * [n, k] as gguf.Model.raw() returns them, parakeet_cuda/gguf.py:135-138)
 * into `packed` (host memory, pq8_packed_size() bytes). */
PQ8_API int pq8_pack_q8_0(const void* gguf_blocks, int n, int k, int layout, void* packed);

/* Pack a [n, k_src] source into columns [k_offset, k_offset + k_src) of a
 * packed [n, k_total] tensor (k_offset and k_src multiples of 32). Used to
 * concatenate the LSTM input and hidden weights along K
 * (decoder.py:58-61 computes W_ih x + W_hh h). The first call on a buffer
 * must have k_offset == 0: it writes the header and zero-fills padding. */
PQ8_API int pq8_pack_q8_0_part(const void* gguf_blocks, int n, int k_src, int k_total, int k_offset,
                       int layout, void* packed);

/* ---- device kernels ------------------------------------------------------ */

/* pq8_pack_q8_0 / pq8_pack_q8_0_part on the device: gguf_blocks are the
 * GGUF bytes already copied to the device (2-byte aligned), packed a device
 * buffer of pq8_packed_size() bytes (16-byte aligned). Same bytes as the host
 * packer once every K part has been written: the k_offset == 0 call writes
 * the header, each call writes all 128 rows (zeros for padding rows) of its
 * K blocks. A later part whose header does not match records PQ8_ERR_LAYOUT
 * in the device status word (pq8_device_status). Replaces the per-layer
 * upload + dequant_q8 of GPU.load_weights (gpu.py:169-184): the raw bytes are
 * copied once and repacked in HBM. */
PQ8_API int pq8_pack_q8_0_device(const void* gguf_blocks, int n, int k, int layout, void* packed, void* stream);
PQ8_API int pq8_pack_q8_0_part_device(const void* gguf_blocks, int n, int k_src, int k_total, int k_offset,
                                      int layout, void* packed, void* stream);

/* Q8_0 -> FP32 expansion, bit-identical to dequant_q8 (runtime.cu:26-33).
 * gguf_blocks: device, n_elements/32 records of 34 bytes; out: device float[n_elements]. */
PQ8_API int pq8_dequant_q8_0(const void* gguf_blocks, float* out, long long n_elements, void* stream);

/* Round n floats (device, 16-byte aligned) to TF32 in place, to nearest with
 * ties away from zero, as the GEMM rounds its operands. A producer that writes
 * activations this way (or a caller that rounds once an input several GEMMs
 * read) lets those GEMMs skip their rounding pass with PQ8_FLAG_X_TF32. */
PQ8_API int pq8_round_tf32(float* x, long long n, void* stream);

/* Tensor-core GEMM (tcgen05, TF32 operands rounded to nearest, FP32 accumulate):
 *   z[m, j] = sum_k x[m, k] * W[j, k]  (+ bias[j]),  y = epilogue(z)
 * Replaces Blas.linear (gpu.py:87-90) + the elementwise epilogue kernels.
 *   w      device, packed ROWS or GLU layout with n rows, k columns
 *   x      device, float[m][k], 16-byte aligned, row stride k
 *   y      device, float[m][out], out = n (ROWS) or n/2 (GLU); may alias resid
 *   bias   device float[n] or NULL
 *   resid  device float[m][out] (EPI_RESIDUAL only)
 * Any m >= 0; k a positive multiple of 32; n >= 1. */
PQ8_API int pq8_gemm(const void* w, const float* x, float* y, const float* bias, const float* resid,
             int m, int n, int k, int epilogue, float alpha, int flags, void* stream);

/* Workspace bytes needed by pq8_gemv / pq8_lstm_layer / pq8_joint_argmax for
 * this shape on the current device. Every workspace starts with a fixed 64 KiB
 * counter area; shapes whose split-K tiles need more counters than it holds
 * (over 16,320 tile x row-group pairs with K split) return
 * PQ8_ERR_UNSUPPORTED_SHAPE. */
PQ8_API int pq8_gemv_workspace_size(int m, int n, int k, size_t* bytes);

/* Zero a workspace before its first use (its counters reset themselves
 * after every call, so this is needed once per buffer; one buffer serves calls
 * of any shape it is large enough for). */
PQ8_API int pq8_workspace_init(void* workspace, size_t bytes, void* stream);

/* HBM-streaming GEMV for the decoder regime, 1 <= m <= PQ8_GEMV_MAX_M:
 * y = epilogue(x @ W^T + bias). Deterministic: fixed summation order
 * (split-K partials are combined in split order by the last CTA).
 * Replaces q8_gemv (runtime.cu:180-188) and the M=1 Blas.linear calls of
 * CUDADecoder (decoder.py:50-52). Arguments as pq8_gemm plus the workspace. */
PQ8_API int pq8_gemv(const void* w, const float* x, float* y, const float* bias, const float* resid,
             int m, int n, int k, int epilogue, float alpha, void* workspace, size_t workspace_bytes,
             void* stream);

/* Dispatch by shape: pq8_gemv for m <= PQ8_LINEAR_GEMV_MAX_M, and for m up
 * to PQ8_GEMV_MAX_M where its FP32 FMA work is small enough to beat the
 * tensor-core GEMM's fixed cost (a measured cost model of both); the
 * tensor-core GEMM otherwise, with split K when its tiles would fill at most
 * half of the SMs (each tile's K blocks shared by 2, 4 or 8 CTAs of one
 * cluster, which exchange their partial sums between their shared memories;
 * each CTA adds 1/S of the tile's rows in split order, so results are
 * deterministic; no workspace is involved). Activations not flagged
 * PQ8_FLAG_X_TF32, 256 rows or more, are rounded to TF32 once into the
 * workspace (one streaming pass, the same bits as rounding inside the GEMM)
 * and the GEMM reads that copy; x itself is not written. The workspace
 * (zeroed once by pq8_workspace_init) must hold
 * pq8_linear_workspace_size(m, n, k) bytes (the GEMV's scratch, and m x k
 * floats after its 64 KiB counter area for that copy); with less, the GEMM
 * rounds the activations itself. PQ8_LINEAR_SPLITS=<s> in the environment
 * forces the split count (1 turns split K off). The drop-in for Blas.linear
 * (gpu.py:87-90). */
PQ8_API int pq8_linear(const void* w, const float* x, float* y, const float* bias, const float* resid,
               int m, int n, int k, int epilogue, float alpha, int flags, void* workspace,
               size_t workspace_bytes, void* stream);
/* Workspace bytes pq8_linear needs for this shape (0 when it needs none). */
PQ8_API int pq8_linear_workspace_size(int m, int n, int k, size_t* bytes);

/* One LSTM layer of the TDT prediction network for m <= PQ8_GEMV_MAX_M streams:
 *   gates = W_ih x + W_hh h + bias, c' = s(f) c + s(i) tanh(g), h' = s(o) tanh(c')
 * W is GATES4-packed [4H, in_k + H] = [W_ih | W_hh] (pq8_pack_q8_0_part twice);
 * bias = b_ih + b_hh (float[4H]). x: float[m][in_k], or, when embed_f16 is
 * not NULL, rows embed_f16[tokens[i]] of an fp16 [vocab][in_k] table
 * (decoder.py:55 looks the embedding up on the host). h, c: float[m][H];
 * h_out, c_out: float[m][H] (must not alias h, c).
 * Replaces 2 Blas.linear + lstm (decoder.py:58-62, runtime.cu:155-163). */
PQ8_API int pq8_lstm_layer(const void* w, const float* x, const uint16_t* embed_f16, const int* tokens,
                   const float* h, const float* c, const float* bias, float* h_out, float* c_out,
                   int m, int hidden, int in_k, void* workspace, size_t workspace_bytes, void* stream);

/* TDT joint for m <= PQ8_GEMV_MAX_M streams: logits = W relu(enc + pred) + bias,
 * then ids[i] = {argmax logits[i][0:vocab), argmax logits[i][vocab:n)} with ties
 * to the lowest index. enc: float[R][k]; row i of the activation uses enc row
 * enc_rows[i] (device int[m]) or, when enc_rows is NULL, row i. pred:
 * float[m][k]; logits: float[m][n], or NULL when only the ids are wanted;
 * ids: int[m][2].
 * Replaces joint_relu + Blas.linear + bias_act + argmax_tdt (decoder.py:66-72,
 * runtime.cu:164-179). */
PQ8_API int pq8_joint_argmax(const void* w, const float* enc, const int* enc_rows, const float* pred,
                             const float* bias, float* logits, int* ids, int m, int n, int k, int vocab,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Commit the candidate LSTM state of the streams whose mask[i] != 0:
 * h[l][i][:] = h_new[l][i][:], c[l][i][:] = c_new[l][i][:] for l < layers.
 * State buffers are float[layers][m][hidden]. decoder.py:74-75 does this by
 * swapping the buffers of its single stream. */
PQ8_API int pq8_tdt_commit(float* h, float* c, const float* h_new, const float* c_new, const int* mask, int m,
                           int layers, int hidden, void* stream);

/* One step of the greedy TDT loop for m <= 1024 streams, on the device. It
 * has no counterpart in the reference, whose loop runs on the host
 * (decoder.py:78-97) and reads the joint's ids back every step; here a decode
 * step is a fixed launch sequence (pq8_lstm_layer x2 + pq8_gemv, then
 * pq8_joint_argmax, pq8_tdt_control, pq8_tdt_commit) that a CUDA graph can
 * replay, with the host polling *remaining now and then.
 * ids: int[m][2] from pq8_joint_argmax (token, duration index); durations:
 * int[n_durations] (model metadata asr.tdt.durations); state: int[m][8] =
 * {frames, t, symbols, previous token, emitted, joint calls, done, 0}, set by
 * the caller to {frames_i, 0, 0, 8192, 0, 0, frames_i == 0, 0} before the
 * first step. Applies the reference's rules (blank 8192; blank with duration 0
 * advances one frame; at most 10 symbols per frame) to the streams not done,
 * then writes the next step's inputs: tokens[i] (predictor input = last
 * emitted token), enc_rows[i] = i * enc_stride + min(t, frames - 1) (row of
 * the next joint call), commit_mask[i] (1 when this step emitted), and
 * *remaining (streams not done). Per joint call it appends {t, token, skip}
 * to trace[i][trace_capacity][3], per emitted token {token, t, skip} to
 * emitted[i][emitted_capacity][3]; a full buffer records PQ8_ERR_WORKSPACE in
 * the device status word instead of writing past it. */
PQ8_API int pq8_tdt_control(const int* ids, const int* durations, int n_durations, int* state, int m,
                            int enc_stride, int* tokens, int* enc_rows, int* commit_mask, int* emitted,
                            int emitted_capacity, int* trace, int trace_capacity, int* remaining, void* stream);

/* pq8_tdt_control followed by pq8_tdt_commit, in one launch (one fewer kernel
 * per decode step; same arguments as the two, hidden a multiple of 4 and the
 * state buffers 16-byte aligned). One difference: the commit takes the
 * candidate state of every stream whose joint token is not blank, including
 * streams already done, whose state no later result reads; pq8_tdt_commit
 * with the mask written by pq8_tdt_control leaves those unchanged. Like
 * pq8_tdt_control it has no counterpart in the reference (decoder.py:74-97
 * runs on the host). */
PQ8_API int pq8_tdt_advance(const int* ids, const int* durations, int n_durations, int* state, int m,
                            int enc_stride, int* tokens, int* enc_rows, int* commit_mask, int* emitted,
                            int emitted_capacity, int* trace, int trace_capacity, int* remaining, float* h,
                            float* c, const float* h_new, const float* c_new, int layers, int hidden, void* stream);

/* One M = 1 product of a GEMV batch: y[0:n'] = epilogue(W x + bias) with W
 * packed [n, k] (GLU-packed for PQ8_EPI_GLU, n' = n / 2; else ROWS, n' = n),
 * x float[k] (16-byte aligned), y float[n'], bias float[n] or NULL, resid
 * float[n'] for PQ8_EPI_RESIDUAL (y = resid + alpha z). */
typedef struct pq8_gemv_task {
  const void* w;
  const float* x;
  float* y;
  const float* bias;
  const float* resid;
  int n, k, epilogue;
  float alpha;
} pq8_gemv_task;

/* Bytes of the plan and of the workspace pq8_gemv_batch_plan needs for these tasks. */
PQ8_API int pq8_gemv_batch_sizes(const pq8_gemv_task* tasks, int count, size_t* plan_bytes,
                                 size_t* workspace_bytes);
/* Many independent M = 1 GEMVs as one launch: the reference runs its M = 1
 * products one q8_gemv launch at a time (runtime.cu:180-188); for matrices of
 * a few MB each, one launch per matrix is bound by launch and ramp-up latency,
 * while here every task's 128-row tiles stream side by side in one grid
 * (each CTA streams up to 32 K blocks of one tile; longer K ranges are split
 * and reduced in split order through the workspace, deterministically).
 * Writes the task table into `plan` (device memory, 16-byte aligned) and
 * zeroes the workspace (device memory, 256-byte aligned; tied to the plan);
 * *ctas receives the grid size for pq8_gemv_batch_run. Synchronises the
 * stream. The tasks' buffers must stay valid while the plan is used. */
PQ8_API int pq8_gemv_batch_plan(const pq8_gemv_task* tasks, int count, void* plan, size_t plan_bytes,
                                void* workspace, size_t workspace_bytes, int* ctas, void* stream);
/* Runs a planned batch (capturable in a CUDA graph; the workspace counters
 * reset themselves, so replays need no re-initialisation). */
PQ8_API int pq8_gemv_batch_run(const void* plan, int ctas, void* stream);

/* Weights of the TDT prediction and joint networks for pq8_tdt_decode, all
 * resident on the device (H = hidden, J = joint width, E = embedding width):
 *   lstm[l]       GATES4-packed [4H, in_l + H] = [W_ih | W_hh], in_0 = E, in_1 = H
 *   lstm_bias[l]  b_ih + b_hh, float[4H] (gate order i, f, g, o)
 *   pred          ROWS-packed joint.pred [J, H]; pred_bias float[J]
 *   joint         ROWS-packed joint.joint_net.2 [n_joint, J]; joint_bias float[n_joint]
 *   embed         fp16 [vocab][E] (decoder.prediction.embed; row 8192 is the blank's)
 * vocab = number of token logits (the rest, n_joint - vocab, are durations). */
typedef struct pq8_tdt_weights {
  const void* lstm[2];
  const float* lstm_bias[2];
  const void* pred;
  const float* pred_bias;
  const void* joint;
  const float* joint_bias;
  const uint16_t* embed;
  int hidden, embed_k, joint_k, n_joint, vocab;
} pq8_tdt_weights;

/* Workspace bytes pq8_tdt_decode needs for m streams. */
PQ8_API int pq8_tdt_decode_workspace_size(int m, int hidden, int joint_k, size_t* bytes);

/* The whole greedy TDT decode of m <= 64 streams in one persistent launch:
 * the loop of decoder.py:78-97 (predict after an emitted token, joint, the
 * control rules of pq8_tdt_control, commit) with no host round trip per step.
 * One CTA per SM keeps its share of all four weights in shared memory for the
 * whole decode; grid barriers (bounded waits: PQ8_ERR_TIMEOUT in the device
 * status word) separate the joint from the prediction-network phases, and the
 * prediction network runs only for streams that emitted.
 * enc: stream i's projected frame t is row i * enc_stride + t of a float[.][J]
 * table. state, emitted, trace: as pq8_tdt_control's (state word 7 holds the
 * stream's committed LSTM slot); set state to {frames_i, 0, 0, 8192, 0, 0,
 * frames_i == 0, 0} for a fresh decode (resume = 0: LSTM state and pred start
 * from zero and the first prediction runs on the blank token). The launch
 * stops when every stream is done or after max_steps joint steps; resume = 1
 * continues such a decode from the workspace (same workspace, state and
 * streams). *steps_out (device int) = joint steps run, *remaining (device
 * int) = streams not done. Results equal the host loop's over pq8_lstm_layer,
 * pq8_gemv and pq8_joint_argmax up to the order of FP32 additions. */
PQ8_API int pq8_tdt_decode(const pq8_tdt_weights* weights, const float* enc, int enc_stride, const int* durations,
                           int n_durations, int* state, int m, int* emitted, int emitted_capacity, int* trace,
                           int trace_capacity, int max_steps, int resume, int* steps_out, int* remaining,
                           void* workspace, size_t workspace_bytes, void* stream);

/* pq8_gemv without a workspace argument, for callers that cannot allocate
 * device memory: a host that keeps all device memory in its own pre-reserved
 * pool, or a latency-critical loop where cudaMalloc would synchronize the
 * device. It has no counterpart in the reference (whose cuBLAS path uses a
 * caller-reserved workspace). Scratch space comes from a fixed 4 MiB array
 * built into the library, held by every GPU that loads the library until the
 * process exits; shapes whose pq8_gemv_workspace_size() exceeds 4 MiB return
 * PQ8_ERR_WORKSPACE. The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) and should come before any stream capture. All calls
 * on a device share the array: calls that overlap on the GPU race, so order
 * them (one stream). Each call clears the array's counters itself, and calls
 * no cudaMalloc/cudaFree. Results equal pq8_gemv's for the same inputs, bit
 * for bit. The array's address (like the status word every entry point uses)
 * is cached per device and does not survive cudaDeviceReset or a release of
 * the primary context: do not call the library on a device after resetting it. */
PQ8_API int pq8_gemv_static(const void* w, const float* x, float* y, const float* bias, const float* resid,
                            int m, int n, int k, int epilogue, float alpha, void* stream);

/* ---- GEMM sequences ----------------------------------------------------------
 * Many pq8_gemm calls as one persistent launch: the encoder issues one
 * Blas.linear per linear per layer (encoder.py:15-36,75-84,115-127 via
 * gpu.py:87-90); here a whole list of them becomes one kernel whose CTAs (one
 * per SM) run the tiles of every GEMM in list order. Tiles of a GEMM start as
 * soon as the 192-row blocks they read are complete, instead of after the
 * previous GEMM has finished everywhere, so neither a launch's ramp-up and
 * drain nor its last partial wave of tiles is paid per GEMM. Each task has
 * pq8_gemm's arguments and meaning, and all tasks of a sequence carry the
 * same PQ8_FLAG_X_TF32 setting; every tile runs the BN = 192 single-CTA
 * configuration. */
typedef struct pq8_gemm_task {
  const void* w;      /* packed Q8_0 weight [n, k] */
  const float* x;     /* activations [m, k], 16-byte aligned */
  float* y;           /* output [m, n] ([m, n/2] for PQ8_EPI_GLU) */
  const float* bias;  /* [n] or NULL */
  const float* resid; /* PQ8_EPI_RESIDUAL: [m, out] (may equal y); else NULL */
  int m, n, k, epilogue;
  float alpha;
  int flags;          /* PQ8_FLAG_X_TF32 | PQ8_FLAG_OUT_TF32 */
  int after;          /* -1, or an earlier task whose output rows this task's x depends on although the
                         buffers do not show it (a LayerNorm or attention run outside the sequence) */
  int after_window;   /* 0: the same rows of `after`; W > 0: all rows of the W-row windows that a tile's
                         rows belong to (e.g. attention over windows of W frames) */
} pq8_gemm_task;

/* Bytes of device memory the plan of `tasks` needs. */
PQ8_API int pq8_sequence_plan_size(const pq8_gemm_task* tasks, int count, size_t* bytes);
/* Lay out the plan of `tasks` in `plan` (device memory, 256-byte aligned):
 * parameters, tensor maps and the dependencies between tasks. Dependencies
 * come from the buffers: a task that reads x or resid rows waits for the last
 * earlier task that wrote them, and a task that writes y waits for the
 * earlier tasks that wrote or read those rows. Buffers are identified by
 * their start address and row width; two that overlap otherwise are refused
 * (PQ8_ERR_UNSUPPORTED_SHAPE), as is a task with more than 4 dependencies of
 * either kind. The plan also holds the tile schedule for this device's SM
 * count: tiles handed out in task order to the CTA a model of the launch frees
 * first (list scheduling with a short lookahead; PQ8_SEQUENCE_SCHEDULE=strided
 * in the environment gives CTA c tiles c, c + SMs, ... instead). Reads each
 * weight's packed header (PQ8_ERR_LAYOUT on a mismatch) and synchronizes
 * `stream`; not for stream capture. The plan stays valid while the buffers
 * and weights it names do, on devices with the same SM count (a run on
 * another records PQ8_ERR_LAYOUT). */
PQ8_API int pq8_sequence_plan(const pq8_gemm_task* tasks, int count, void* plan, size_t plan_bytes, void* stream);
/* Run a plan: one launch (one CTA per SM) that computes every task. Runs of
 * one plan must not overlap on the GPU (its completion counters are shared and
 * reset by each run's last CTA). A dependency wait that expires records
 * PQ8_ERR_TIMEOUT (pq8_device_status); the plan is then to be made again. */
PQ8_API int pq8_sequence_run(const void* plan, void* stream);

/* Read and clear the device-side status word that kernels set on a layout
 * mismatch or an expired bounded wait. Synchronizes `stream`. *status = 0 or
 * PQ8_ERR_LAYOUT / PQ8_ERR_TIMEOUT. */
PQ8_API int pq8_device_status(int* status, void* stream);

/* ---- the FastConformer block around the linears ----------------------------
 * The rest of one encoder block (parakeet_cuda/reference.py:33-66) on the
 * device: with these and pq8_gemm, a whole block runs without the host. */

/* LayerNorm of rows of `width` floats (multiple of 128, at most 1024), eps
 * 1e-5: y = (x - mean) / sqrt(var + eps) * w + b. PQ8_FLAG_OUT_TF32 rounds y
 * to TF32 for a following pq8_gemm with PQ8_FLAG_X_TF32. All pointers 16-byte
 * aligned. Replaces layer_norm (runtime.cu:38-48). */
PQ8_API int pq8_layer_norm(const float* x, const float* w, const float* b, float* y, int rows, int width,
                           int flags, void* stream);

/* Conv-module middle (reference.py:60-63): depthwise convolution with 9 taps
 * along the frames of each of `windows` windows of `t` frames (zero rows
 * beyond a window's ends), BatchNorm with running statistics (eps 1e-5),
 * SiLU. x, y: float[windows * t][channels] (distinct, 16-byte aligned);
 * w9_f16: the GGUF fp16 depthwise weight [channels][9]; bn_*: float[channels].
 * Replaces depthwise1 (runtime.cu:63-71). */
PQ8_API int pq8_conv_depthwise_bn_silu(const float* x, const uint16_t* w9_f16, const float* bn_weight,
                                       const float* bn_bias, const float* bn_mean, const float* bn_var, float* y,
                                       int windows, int t, int channels, int flags, void* stream);

/* Relative-position self-attention of 8 heads x 128 over `windows` windows of
 * `t` frames (reference.py:46-57). qkv: float[windows * t][3072] (Q | K | V,
 * the packed linear_q/k/v output); pos: float[2t - 1][1024], linear_pos of
 * the positional rows pe[limit - t : limit + t - 1], shared by all windows;
 * pos_bias_u / _v: float[1024] (head-major); ctx: float[windows * t][1024],
 * heads merged. Scores ((q + u) k + (q + v) p_{t-1+j-i}) / sqrt(128), softmax
 * over keys, context = probabilities x V. By default one fused kernel does
 * everything on chip (tcgen05 products with FP16 operands, which keep TF32's
 * 11-bit significand, FP32 accumulation in tensor memory, online softmax;
 * a CTA per window, head and 128 queries); with
 * PQ8_FLAG_FP32_PRODUCTS the three products are FP32 cuBLAS GEMMs around pq8
 * bias / shift / softmax kernels (an exactness reference, slower).
 * PQ8_FLAG_OUT_TF32 rounds ctx for linear_out. Replaces query_bias, rel_scores, softmax and the attention
 * GEMMs of encoder.py:95-112 (runtime.cu:115-137). */
PQ8_API int pq8_attention_workspace_size(int windows, int t, size_t* bytes);
PQ8_API int pq8_rel_attention(const float* qkv, const float* pos, const float* pos_bias_u, const float* pos_bias_v,
                              float* ctx, int windows, int t, int flags, void* workspace, size_t workspace_bytes,
                              void* stream);

/* Subsampling stem (reference.py:11-30, encoder.py:38-66) for `windows`
 * windows of `frames` mel frames: mel float[windows][frames][128]. Three
 * 3x3 stride-2 stages (full convolution to 256 channels + ReLU; twice
 * depthwise + pointwise 256 x 256 + ReLU), flattened channel-major to 4096 and
 * projected by the Q8_0 output linear: out float[windows * t][1024] with
 * t = ceil(ceil(ceil(frames / 2) / 2) / 2) rows per window. w0, w2, w5:
 * float[256][9] (the GGUF's fp16 kernels as float); w3, w6: float[256][256]
 * (output channel major, 16-byte aligned); b*: float[256]; w_out: packed Q8_0
 * [1024, 4096] (ROWS), b_out: float[1024]. The pointwise products run on the
 * pq8 tensor-core kernel with the FP32 weights rounded to TF32 (with
 * PQ8_FLAG_FP32_PRODUCTS: FP32 cuBLAS products, an exactness reference);
 * everything else is pq8 kernels and pq8_gemm. Replaces conv_first, conv_dw2,
 * the stem SGEMMs, bias_act and flatten_stem (runtime.cu:73-101). */
PQ8_API int pq8_stem_workspace_size(int windows, int frames, size_t* bytes);
PQ8_API int pq8_stem(const float* mel, int windows, int frames, const float* w0, const float* b0, const float* w2,
                     const float* b2, const float* w3, const float* b3, const float* w5, const float* b5,
                     const float* w6, const float* b6, const void* w_out, const float* b_out, float* out, int flags,
                     void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* PQ8_H */
