/*
 * apex_attn — C ABI of the B200 (sm_100a) fused attention forward and backward.
 *
 * This header is the drop-in boundary for the operator
 *   custom_attention_forward(q, k, v, causal=True, sm_scale=None) -> o
 * of mls-bench_fused_attention/fused_attention.py:155-193 (identical copy at
 * submission.py:179-217); apex_attn_bwd adds the backward that training callers need. The Python host module `apex_attn` binds it with ctypes;
 * any other FFI binds the same symbols.
 *
 * Conventions: all pointers are device pointers on one CUDA device, tensors are
 * logical [B, H, N, D] with unit stride along D, strides are given in elements.
 * Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 * stream).
 *
 * Device-side errors are sticky. When a kernel of this library records a device-side
 * error (a bounded wait expired, so its outputs are incomplete), it also sets a flag in
 * mapped pinned host memory. Every forward and backward entry point reads that flag
 * before it launches anything and returns APEX_ATTN_ERR_DEVICE_TIMEOUT while it is set,
 * until apex_attn_device_status() reads and clears the device's state. No call
 * synchronises for this: the first call that starts after the failing kernel wrote the
 * flag reports it (the allocation-free entry point has its own reader, below). No call allocates caller-visible memory; the library keeps one small
 * scratch buffer per device (a status word for device-side error reporting and the
 * work-item counters of its scheduler).
 */
#ifndef APEX_ATTN_H_
#define APEX_ATTN_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (returned by every entry point; 0 = success). */
#define APEX_ATTN_OK 0
#define APEX_ATTN_ERR_INVALID_ARGUMENT -1   /* null pointer, non-positive size */
#define APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM -2
#define APEX_ATTN_ERR_UNSUPPORTED_DTYPE -3
#define APEX_ATTN_ERR_BAD_LAYOUT -4         /* stride/alignment not TMA-compatible */
#define APEX_ATTN_ERR_BAD_SCALE -5          /* sm_scale not finite and > 0 */
#define APEX_ATTN_ERR_NO_DEVICE -6          /* pointer not on a CUDA device / no device */
#define APEX_ATTN_ERR_UNSUPPORTED_ARCH -7   /* device is not sm_100 */
#define APEX_ATTN_ERR_TENSOR_MAP -8         /* cuTensorMapEncodeTiled rejected a tensor */
#define APEX_ATTN_ERR_LAUNCH -9             /* kernel launch failed */
#define APEX_ATTN_ERR_DEVICE_TIMEOUT -10    /* a kernel hit its bounded-wait limit (sticky, below) */
#define APEX_ATTN_ERR_TOO_LARGE -11         /* sizes exceed the supported range */
#define APEX_ATTN_ERR_CUDA -12              /* other CUDA runtime error */

/* Element types. */
#define APEX_ATTN_BF16 0
#define APEX_ATTN_FP16 1

/*
 * Causal (or full) attention forward:
 *   o[b,h,i,:] = sum_j softmax_j(q[b,h,i,:] . k[b,h,j,:] * sm_scale) v[b,h,j,:]
 * with j <= i when causal != 0. Accumulation is fp32; o has the input dtype.
 * lse (nullable) receives the fp32 natural-log logsumexp of each row, contiguous
 * [B, H, N].
 *
 * strides: 12 values, element strides (batch, head, seq) for q, k, v, o in that
 * order. Each must be a multiple of 8 elements (16 bytes); pointers 16-byte aligned.
 * head_dim: 64, 128 or 256 (fused_attention.py:148-152 covers the same three).
 *
 * Replaces: custom_attention_forward body, fused_attention.py:155-193, and the
 * per-head-dim table _CONFIGS, fused_attention.py:148-152 (a KeyError there is
 * APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM here).
 */
int apex_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                  int heads, int seqlen, int head_dim, int dtype, int causal, float sm_scale,
                  const long long* strides, void* stream);

/*
 * Extended forward: the operation of apex_attn_fwd plus grouped-query attention and a
 * causal sliding window, with the arguments in a struct.
 *   heads_kv     K/V heads; heads_q % heads_kv == 0, query head h reads K/V head
 *                h / (heads_q / heads_kv). k and v are [B, heads_kv, N, D].
 *   window_left  -1: no window. >= 0 (causal only): row i sees keys j with
 *                i - window_left <= j <= i.
 *   strides      as for apex_attn_fwd (k and v strides refer to their heads_kv heads).
 * Returns APEX_ATTN_ERR_INVALID_ARGUMENT for heads_q % heads_kv != 0, window_left < -1,
 * or a window without causal. No counterpart in the reference operator; it covers the
 * attention call of the reference's nanochat model (flash_attn_func with GQA and
 * window_size, nanochat_autoresearch/solutions/train.py:690-719).
 */
typedef struct apex_attn_fwd_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse; /* nullable */
  int batch;
  int heads_q;
  int heads_kv;
  int seqlen;
  int head_dim;
  int dtype;
  int causal;
  int window_left;
  float sm_scale;
  long long strides[12];
} apex_attn_fwd_args;

int apex_attn_fwd_ex(const apex_attn_fwd_args* args, void* stream);

/*
 * Packed variable-length forward: the operation of apex_attn_fwd_ex on a batch of
 * sequences of different lengths stored back to back (flash-attn's varlen layout).
 *   q, o         [total, heads_q, D];   k, v  [total, heads_kv, D]
 *   cu_seqlens   device int32 [batch + 1]: sequence b is rows [cu[b], cu[b+1]), cu[0] = 0,
 *                nondecreasing, cu[batch] = total (the same offsets for q and k/v: packed
 *                self-attention). Offsets are clamped to [0, total] and lengths to
 *                max_seqlen on the device, so a malformed array gives wrong rows, never an
 *                out-of-bounds access.
 *   max_seqlen   the longest sequence (sizes the schedule; longer sequences are cut).
 *   lse          nullable, fp32 [heads_q, total].
 *   strides      8 values: (token, head) element strides of q, k, v, o.
 * Rows of o outside every sequence are not written. Causal, window_left, GQA and sm_scale
 * as for apex_attn_fwd_ex; the mask is relative to each sequence's first row.
 * Has no counterpart in the reference operator (the GQA/varlen row of its next steps).
 */
typedef struct apex_attn_varlen_args {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse; /* nullable */
  const int* cu_seqlens;
  int batch;
  int heads_q;
  int heads_kv;
  int total;
  int max_seqlen;
  int head_dim;
  int dtype;
  int causal;
  int window_left;
  float sm_scale;
  long long strides[8];
} apex_attn_varlen_args;

int apex_attn_fwd_varlen(const apex_attn_varlen_args* args, void* stream);

/*
 * Selects the forward kernel for later calls in this process (all devices):
 *   0  automatic (default): for batched calls at head dim 128 without a window, the tile
 *      kernel (one 128-row query tile per CTA, S and P double-buffered in tensor memory,
 *      TMA-store epilogue) when the call has fewer than 3 x (SM count) 256-row query
 *      items (batch x heads x ceil(N / 256)), or N <= 2048 and fewer than 8 x (SM count);
 *      the two-sub-tile kernel for every other call (measured crossovers on B200);
 *   1  the two-sub-tile kernel for every call;
 *   2  the tile kernel wherever it applies (batched, head dim 64 or 128, no window).
 * Both kernels compute the same function within the stated tolerances; this exists to
 * measure them against each other. Returns APEX_ATTN_ERR_INVALID_ARGUMENT for other values.
 * No counterpart in the reference (its _CONFIGS table picks one kernel per head dim,
 * fused_attention.py:148-152).
 */
int apex_attn_set_forward_kernel(int kind);

/*
 * Reports which forward kernel a call of these dimensions runs under the current
 * selection (apex_attn_set_forward_kernel) on a device with `num_sms` SMs: 1 = the
 * two-sub-tile kernel, 2 = the tile kernel. `window` is -1 for none; `packed` != 0 for a
 * packed batch (apex_attn_fwd_varlen), whose `batch` is the sequence count and `seq_len`
 * the longest sequence. Launches nothing and needs no device. Returns
 * APEX_ATTN_ERR_INVALID_ARGUMENT for non-positive sizes or SM count, window < -1, or a
 * head dim other than 64, 128 or 256. No counterpart in the reference.
 */
int apex_attn_forward_kernel_for(int batch, int heads, int seq_len, int head_dim, int window,
                                 int packed, int num_sms);

/*
 * Reads and clears the device status word of `device` after synchronising that
 * device, and clears the sticky host flag. *flags receives the raw bits (1 = a kernel hit its bounded-wait limit,
 * 2 = a copy or MMA still in flight at kernel teardown did not land within the limit,
 * 4 = the dynamic shared-memory base was not 1 KB aligned, so a kernel did nothing).
 * Returns APEX_ATTN_ERR_DEVICE_TIMEOUT when any bit was set.
 * Has no counterpart in the reference (its Triton kernels cannot report device faults).
 */
int apex_attn_device_status(int device, int* flags);

/*
 * Launches a one-CTA kernel whose bounded wait on an mbarrier that nothing arrives
 * on must expire after `timeout_us` microseconds, setting the device status bit.
 * Used by the failure-detection test; it never faults or hangs the GPU.
 * Has no counterpart in the reference.
 */
int apex_attn_selftest_wait_timeout(int timeout_us, void* stream);

/*
 * Allocation-free form of apex_attn_fwd: same arguments, same kernel, same results.
 * No counterpart in the reference; it exists for callers that cannot call cudaMalloc
 * (a process whose device memory is owned by a pool or a serving runtime, a plugin in a
 * host that forbids allocations outside its own allocator, a real-time loop).
 *
 * The caller passes the inputs and outputs as for apex_attn_fwd. The kernel's scratch
 * (a 4-byte device status word and a 4-byte work-item counter, one of 32 that rotate
 * between calls) lives in a fixed 256-byte static device array of the library that every
 * device loading the library holds until process exit; this entry point calls no
 * cudaMalloc, cudaFree or other allocating routine. The scratch need does not grow with
 * B, H, N or D; sizes outside the kernel's supported range are rejected with
 * APEX_ATTN_ERR_TOO_LARGE.
 *
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 * and sets kernel attributes for that device, so make it before any stream capture.
 * Each call clears the status word and its counter on `stream` before its kernel. All
 * calls share the array: calls that overlap on the GPU (other streams, other threads)
 * race on the status word, and on a counter once more than 32 calls are in flight. A
 * bounded wait that expires still ends the kernel early; its status bit stays in the
 * shared scratch until the next allocation-free call clears it, and only
 * apex_attn_noalloc_status reads it (apex_attn_device_status does not). This path keeps
 * no sticky host flag, since that needs pinned host memory.
 */
int apex_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                          int batch, int heads, int seqlen, int head_dim, int dtype, int causal,
                          float sm_scale, const long long* strides, void* stream);

/*
 * Reads and clears the status word that apex_attn_fwd_noalloc launches on `device` share,
 * after synchronising the device; allocates nothing. *flags receives the bits described
 * for apex_attn_device_status; returns APEX_ATTN_ERR_DEVICE_TIMEOUT when any was set. The
 * word holds only what happened since the last allocation-free call began (each call
 * clears it before its kernel), so read it after the call whose outcome matters and
 * before the next one. No counterpart in the reference.
 */
int apex_attn_noalloc_status(int device, int* flags);

/*
 * Backward of the attention computed by apex_attn_fwd / apex_attn_fwd_ex:
 *   dq = d(sum o * dout)/dq, dk, dv likewise, for the same causal / window_left / grouped-
 *   query settings. Inputs: q, k, v, the forward output o, the upstream gradient dout (all
 *   of the input dtype) and the forward's fp32 natural-log logsumexp lse (contiguous
 *   [B, heads_q, N], as apex_attn_fwd writes it). Outputs dq [B, heads_q, N, D] and dk, dv
 *   [B, heads_kv, N, D] in the input dtype; grouped-query heads sum into their K/V head.
 *
 * strides: 24 values, element strides (batch, head, seq) of q, k, v, o, dout, dq, dk, dv in
 * that order; the rules of apex_attn_fwd apply to each (unit head-dim stride, multiples of
 * 8 elements, 16-byte aligned pointers), so [B, N, H, D] views need no copy.
 * head_dim: 64 or 128 (else APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM).
 * workspace: device memory of at least apex_attn_bwd_workspace_bytes(batch, heads_q,
 * seqlen) bytes, 16-byte aligned, on the same device; used only during the call (it holds
 * two fp32 values per query row). Smaller: APEX_ATTN_ERR_INVALID_ARGUMENT.
 * Asynchronous on `stream`; results are deterministic (no atomics). apex_attn_bwd_mode
 * selects the faster fused algorithm instead.
 *
 * Replaces: _flash_attn_bwd(q, k, v, out, grad_output, lse, causal=True,
 * window_size_left=w), the backward that nanochat's attention custom op calls
 * (nanochat_autoresearch/solutions/train.py:491,508-519).
 */
typedef struct apex_attn_bwd_args {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  void* dq;
  void* dk;
  void* dv;
  int batch;
  int heads_q;
  int heads_kv;
  int seqlen;
  int head_dim;
  int dtype;
  int causal;
  int window_left;
  float sm_scale;
  long long strides[24];
} apex_attn_bwd_args;

/* Bytes of workspace apex_attn_bwd needs (0 for non-positive sizes). */
size_t apex_attn_bwd_workspace_bytes(int batch, int heads_q, int seqlen);

int apex_attn_bwd(const apex_attn_bwd_args* args, void* workspace, size_t workspace_bytes,
                  void* stream);

/*
 * Backward algorithms (the `mode` of apex_attn_bwd_mode / apex_attn_bwd_varlen_mode):
 *   APEX_ATTN_BWD_DETERMINISTIC  what apex_attn_bwd runs: a dK/dV pass and a dQ pass that
 *                                recomputes the scores; bitwise reproducible.
 *   APEX_ATTN_BWD_FUSED          one pass: each (key block, query tile) step also computes
 *                                its dQ tile and adds it into an fp32 accumulator in the
 *                                workspace with global reductions, then a cast writes dq.
 *                                Five GEMMs per step instead of seven; dk and dv are
 *                                bitwise the same as in the deterministic mode, dq is not
 *                                reproducible bit for bit (the reductions' order varies).
 * Any other mode: APEX_ATTN_ERR_INVALID_ARGUMENT.
 */
#define APEX_ATTN_BWD_DETERMINISTIC 0
#define APEX_ATTN_BWD_FUSED 1

/* Workspace bytes for `mode` (0 for non-positive sizes). The fused mode adds an fp32
 * accumulator of batch * heads_q * seqlen * head_dim values; for a packed batch pass
 * max_seqlen as seqlen. */
size_t apex_attn_bwd_workspace_bytes_mode(int batch, int heads_q, int seqlen, int head_dim, int mode);

/* apex_attn_bwd with the algorithm chosen by `mode`; workspace as
 * apex_attn_bwd_workspace_bytes_mode(batch, heads_q, seqlen, head_dim, mode). */
int apex_attn_bwd_mode(const apex_attn_bwd_args* args, int mode, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Backward of apex_attn_fwd_varlen: dq, dk, dv of a packed variable-length batch.
 *   q, o, dout, dq   [total, heads_q, D];   k, v, dk, dv   [total, heads_kv, D]
 *   lse              fp32 [heads_q, total], as apex_attn_fwd_varlen writes it
 *   cu_seqlens, max_seqlen, causal, window_left, sm_scale: as for apex_attn_fwd_varlen
 *   strides          16 values: (token, head) element strides of q, k, v, o, dout, dq, dk, dv
 *   workspace        apex_attn_bwd_workspace_bytes(batch, heads_q, max_seqlen) bytes
 * Rows outside every sequence are not written. Offsets are clamped on the device as for
 * the forward. Head dims 64 and 128. No counterpart in the reference operator.
 */
typedef struct apex_attn_bwd_varlen_args {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  void* dq;
  void* dk;
  void* dv;
  const int* cu_seqlens;
  int batch;
  int heads_q;
  int heads_kv;
  int total;
  int max_seqlen;
  int head_dim;
  int dtype;
  int causal;
  int window_left;
  float sm_scale;
  long long strides[16];
} apex_attn_bwd_varlen_args;

int apex_attn_bwd_varlen(const apex_attn_bwd_varlen_args* args, void* workspace,
                         size_t workspace_bytes, void* stream);

/* apex_attn_bwd_varlen with the algorithm chosen by `mode` (see apex_attn_bwd_mode);
 * workspace as apex_attn_bwd_workspace_bytes_mode(batch, heads_q, max_seqlen, head_dim,
 * mode). The fused mode needs total <= batch * max_seqlen (true of any valid cu_seqlens),
 * else APEX_ATTN_ERR_INVALID_ARGUMENT. */
int apex_attn_bwd_varlen_mode(const apex_attn_bwd_varlen_args* args, int mode, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Number of SMs of `device` (the persistent kernels' grid is min(work items, this)), or a
 * negative status: APEX_ATTN_ERR_NO_DEVICE for a bad ordinal or no device,
 * APEX_ATTN_ERR_UNSUPPORTED_ARCH if it is not sm_100. Lets a caller size its own batching
 * (e.g. how many heads make a full wave). No counterpart in the reference. */
int apex_attn_num_sms_hint(int device);

/* Human-readable text for a status code. Replaces the exception text the reference
 * harness prints on failure (submission.py:299-306). */
const char* apex_attn_strerror(int status);

/* Library version as major*10000 + minor*100 + patch. */
int apex_attn_version(void);

/* 1 if head_dim is supported by apex_attn_fwd, else 0 (mirrors `headdim in _CONFIGS`,
 * fused_attention.py:148-152). */
int apex_attn_supports_head_dim(int head_dim);

#ifdef __cplusplus
}
#endif

#endif /* APEX_ATTN_H_ */
