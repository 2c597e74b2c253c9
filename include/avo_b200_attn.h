/*
 * avo_b200_attn.h - C ABI of the B200 (sm_100a) attention-forward library
 * libavo_b200_attn.so.
 *
 * The AVO candidate contract is the Python callable `attention(q, k, v, causal)`
 * (reference: candidates/torch_sdpa_seed.py:6-7, loaded and checked by
 * avo/benchmark.py:406-418); the reference's CUDA seeds reach their kernels through
 * a pybind11 binding `attention(q, k, v, causal)` that TORCH_CHECKs its tensors and
 * calls `attention_cuda` (candidates/cuda_mma_attention/attention.cpp:8-26,
 * candidates/cuda_mma_attention/attention_kernel.cu:175-206).  This header is the
 * replacement boundary: plain pointers and sizes, no torch types.  Tensors are
 * caller-owned device memory; nothing here allocates device memory; every launch is
 * asynchronous on `stream` (a cudaStream_t, 0 = legacy default stream).
 *
 * Layout: q, k, v, o are bf16 [batch, heads, seq, 128] contiguous (the SDPA layout);
 * lse is fp32 [batch, heads, seq], natural log of sum_j exp(scale * q.k_j).
 *
 * Return codes (host side, synchronous):
 *   AVO_B200_OK                0
 *   AVO_B200_EINVAL            1  bad argument (shape, alignment, null pointer, scale)
 *   AVO_B200_ENODEV            2  current device is not compute capability 10.0 (B200)
 *   AVO_B200_ELAUNCH           3  CUDA reported an error at launch
 *   AVO_B200_ETENSORMAP        4  cuTensorMapEncodeTiled rejected a descriptor
 *   AVO_B200_EDRIVER           5  driver entry point for tensor maps unavailable
 *   AVO_B200_ETOOBIG           6  problem exceeds the static scratch of the no-allocation entry
 *   AVO_B200_EREGS             7  the built kernel's register allocation is not the one its
 *                                 per-warpgroup register split (setmaxnreg) was computed for; the
 *                                 library was built by a compiler that allocated differently and
 *                                 refuses to launch (rebuild with the nvcc this file was tuned on)
 *
 * Device status bits (written asynchronously into *status_dev when non-null; the
 * caller zeroes the word and reads it after synchronizing):
 *   AVO_B200_STATUS_WATCHDOG   1  a pipeline wait exceeded the watchdog; outputs invalid
 *   AVO_B200_STATUS_DRAIN      2  draining in-flight work after an abort also timed out
 */
#ifndef AVO_B200_ATTN_H_
#define AVO_B200_ATTN_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AVO_B200_OK 0
#define AVO_B200_EINVAL 1
#define AVO_B200_ENODEV 2
#define AVO_B200_ELAUNCH 3
#define AVO_B200_ETENSORMAP 4
#define AVO_B200_EDRIVER 5
#define AVO_B200_ETOOBIG 6
#define AVO_B200_EREGS 7

/* Row capacity (batch * heads * seq) of avo_b200_attn_fwd_split_noalloc's scratch. */
#define AVO_B200_NOALLOC_MAX_ROWS 16384
#define AVO_B200_NOALLOC_MAX_SPLITS 64

#define AVO_B200_STATUS_WATCHDOG 1
#define AVO_B200_STATUS_DRAIN 2

/* ABI revision of this header; bumped on any signature change. */
int avo_b200_abi_version(void);

/* Human-readable text for a return code. */
const char* avo_b200_strerror(int code);

/*
 * Full attention forward, the drop-in for the candidate's `attention()`
 * (candidates/cuda_mma_attention/attention_kernel.cu:175-206 `attention_cuda`, and the
 * guard it enforces, D == 128).  o = softmax(softmax_scale * q k^T [+ causal mask]) v.
 * causal != 0 masks key j > query i (candidates/cuda_naive_attention/attention_kernel.cu:28).
 * lse may be null.  seq >= 1 (any length; ragged tails are masked), head_dim == 128,
 * softmax_scale > 0 (the reference uses 1/sqrt(head_dim), attention_kernel.cu:198).
 */
int avo_b200_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                      int heads, int seq, int head_dim, int causal, float softmax_scale,
                      int* status_dev, void* stream);

/*
 * Bytes of workspace avo_b200_attn_fwd_ws wants on the current device (it grows with the
 * multiprocessor count: about 38.5 MB on a 148-SM B200).  No reference counterpart.
 */
int avo_b200_attn_workspace_size(size_t* bytes);

/*
 * avo_b200_attn_fwd with caller-provided scratch (a workspace, as cuDNN and
 * FlashAttention take one; no reference counterpart: the reference's single-GPU seeds
 * need none).  With it the kernel may cut a work item's key/value range between CTAs
 * (stream-K) where whole items would leave multiprocessors idle, e.g. one GPU's head
 * shard of a problem split over 8 GPUs; the pieces are merged by log-sum-exp inside the
 * same launch
 * (a cooperative launch: all CTAs resident).  Same arguments and results as
 * avo_b200_attn_fwd otherwise.  workspace: device memory of at least
 * avo_b200_attn_workspace_size() bytes, 256-byte aligned, ZERO-FILLED before its first
 * use; every launch that completes leaves it zeroed again, so it is reused as is, but
 * after a watchdog abort it must be zeroed again.  Launches that share one workspace
 * must not overlap in time.  workspace == NULL behaves exactly like avo_b200_attn_fwd.
 */
int avo_b200_attn_fwd_ws(const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                         int heads, int seq, int head_dim, int causal, float softmax_scale, void* workspace,
                         size_t workspace_bytes, int* status_dev, void* stream);

/*
 * Diagnostic (no reference counterpart; host only, needs no GPU): the work plan the
 * kernel would run for these sizes on `sm_count` multiprocessors, with (split != 0) or
 * without a workspace.  plan_out[4] = {mode (0 whole items in waves, 1 waves + split
 * tail, 2 causal whole items in host-built per-CTA lists over groups of heads), CTAs,
 * shortest split run in tiles (mode 1) or pairs per group (mode 2), items in waves}.  If units and counts are
 * non-null, CTA c's units go to units[(c * max_units + n) * 8 ...] as
 * {bh, q0, t0, t1, kind (0 whole, 1 first piece, 2 continuation), segment, first and
 * last CTA holding continuation pieces} and counts[c] = its number of units (only the
 * first max_units are stored).
 */
int avo_b200_schedule_units(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0, long long kv_pos0,
                            int sm_count, int split, int* plan_out, int* units, int max_units, int* counts);

/*
 * Block form used by the context-parallel ring (no reference counterpart: the
 * reference is single-GPU, avo/benchmark.py:212).  Attention of num_bh heads of
 * seq_q query rows against seq_kv key/value rows, each head `*_head_stride`
 * elements apart (rows are 128 elements, contiguous).  The causal mask compares
 * sequence positions: key row r sits at kv_pos0 + r, query row r at q_pos0 + r.
 * Writes normalized o (bf16) and lse (fp32, may be null); rows that see no key get
 * o = 0 and lse = -inf.  Strides must be multiples of 8 elements.
 */
int avo_b200_attn_fwd_block(const void* q, const void* k, const void* v, void* o, float* lse,
                            int num_bh, int seq_q, int seq_kv, int head_dim,
                            long long q_head_stride, long long kv_head_stride,
                            long long o_head_stride, long long lse_head_stride, int causal,
                            float softmax_scale, long long q_pos0, long long kv_pos0,
                            int* status_dev, void* stream);

/*
 * Merge one partial result into a running fp32 accumulator by log-sum-exp
 * (ring context parallelism; no reference counterpart).  For each of num_bh heads
 * and `rows` rows:  lse' = log(exp(acc_lse) + exp(part_lse)),
 *                   acc_o' = acc_o * exp(acc_lse - lse') + part_o * exp(part_lse - lse').
 * acc_o fp32 and part_o bf16 are [num_bh, rows, 128] with contiguous 128-element rows
 * and the given head strides (elements); acc_lse and part_lse are fp32 [num_bh, rows]
 * with contiguous rows and the given head strides.  An accumulator row with
 * acc_lse = -inf takes the partial as is (its acc_o contents are ignored).
 */
int avo_b200_lse_merge(float* acc_o, float* acc_lse, const void* part_o, const float* part_lse,
                       int num_bh, int rows, int head_dim, long long acc_o_head_stride,
                       long long acc_lse_head_stride, long long part_o_head_stride,
                       long long part_lse_head_stride, void* stream);

/*
 * Convert a merged fp32 accumulator to the bf16 output: out[h, r, :] = acc_o[h, r, :],
 * both [num_bh, rows, 128] with contiguous rows and the given head strides (elements).
 */
int avo_b200_acc_to_bf16(const float* acc_o, void* out, int num_bh, int rows, int head_dim,
                         long long acc_head_stride, long long out_head_stride, void* stream);

/*
 * Attention forward with the same arguments, layout and result as avo_b200_attn_fwd,
 * computed as n_splits consecutive key/value blocks (whole 128-key tiles each) whose
 * partial O and LSE are merged by log-sum-exp, using ONLY scratch the library holds in
 * file-scope static device arrays: it allocates nothing (no cudaMalloc, no allocating
 * library routine) and needs no workspace argument.  No counterpart in the reference.
 *
 * Limit: batch * heads * seq <= AVO_B200_NOALLOC_MAX_ROWS (16384 rows, about 12 MiB of
 * static scratch per device); larger problems return AVO_B200_ETOOBIG before any device
 * work.  1 <= n_splits <= AVO_B200_NOALLOC_MAX_SPLITS.  The scratch is shared by every
 * caller on a device: calls that overlap in time (different streams, threads or
 * processes' concurrent use of one library instance) race on it and must be
 * serialized by the caller.  Partial results pass through bf16, so outputs may differ
 * from avo_b200_attn_fwd by bf16 rounding.
 */
int avo_b200_attn_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                                    int batch, int heads, int seq, int head_dim, int causal,
                                    float softmax_scale, int n_splits, int* status_dev, void* stream);

/*
 * Self-test of the device watchdog without faulting the GPU: one CTA waits on an
 * mbarrier that nothing ever completes, with the given limit in microseconds; the
 * wait expires, the kernel sets AVO_B200_STATUS_WATCHDOG in *status_dev and returns.
 */
int avo_b200_watchdog_selftest(int timeout_us, int* status_dev, void* stream);

/*
 * Diagnostic (no reference counterpart): y[i] = the softmax's FMA-pipe 2^x[i] for
 * x[i] in [-125, 127], computed by the same device function the attention kernel uses
 * for part of its exponentials (degree-3 relative-minimax polynomial after a
 * Cody-Waite split; relative error < 7.5e-5).  x and y are fp32 device arrays of n
 * elements.  Exists so tests can compare it with CUDA's exp2f on the device.
 */
int avo_b200_exp2_poly_eval(const float* x, float* y, long long n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AVO_B200_ATTN_H_ */
