/*
 * C ABI of the B200 (sm_100a) causal depthwise conv1d library, libcausal_conv1d_b200.so.
 *
 *   out[b, t, d] = act(bias[d] + sum_k weight[d, k] * x[b, t - (W - 1) + k, d])
 *
 * over channels-last inputs x (B, T, D). Rows t < 0 read initial_states (B, W-1, D) or zero;
 * seq_idx (B, T) int32 packs several sequences per row (taps never cross a sequence boundary and
 * rows with a negative id are padding whose output is 0); act is identity or SiLU.
 *
 * These entry points replace the kernel launches of the reference implementation,
 * jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py, one for one. The
 * argument lists carry what those launches pass (device pointers, the (B, T, D, W) sizes, the
 * batch/time strides of x and dout in elements, the presence flags as null/non-null pointers)
 * plus the element types the Triton JIT would read off the tensors and the CUDA stream that
 * torch's current stream supplies there.
 *
 * Conventions for every entry point:
 *  - All pointers are device pointers on the current CUDA device; the work is enqueued on
 *    `stream` (a cudaStream_t; NULL is the legacy default stream). cc1d_fwd and cc1d_bwd allocate
 *    nothing and never synchronise the host, so they can be captured in a CUDA graph.
 *  - The channel stride of x and dout is 1. out, dx, final_states, dinit, initial_states and
 *    dfinal_states are contiguous. weight is (D, W) row-major, bias is (D).
 *  - Element type codes: CC1D_F32, CC1D_F16, CC1D_BF16. out, final_states, dx and
 *    dfinal_states have the type of x; dinit has the type of initial_states; dweight and dbias
 *    have the types of weight and bias.
 *  - Return value 0 on success, else one of CC1D_ERR_*; cc1d_error_string() describes it.
 */
#ifndef CAUSAL_CONV1D_B200_H_
#define CAUSAL_CONV1D_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { CC1D_F32 = 0, CC1D_F16 = 1, CC1D_BF16 = 2 };

enum {
  CC1D_OK = 0,
  CC1D_ERR_INVALID = 1,     /* bad size, stride, dtype code or missing required pointer */
  CC1D_ERR_UNSUPPORTED = 2, /* width above the largest supported (256) */
  CC1D_ERR_WORKSPACE = 3,   /* workspace smaller than cc1d_bwd_workspace_bytes() */
  CC1D_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed; see cc1d_last_cuda_error() */
  CC1D_ERR_SCRATCH_LIMIT = 5, /* cc1d_bwd_noalloc: problem needs more than its fixed scratch */
  CC1D_ERR_LAYOUT = 6         /* cc1d_bwd_split: pieces or dx strides outside its fast path */
};

/* Interface version of this header; bumped on any signature change. */
int cc1d_abi_version(void);

/*
 * Forward. Replaces the `_fwd_kernel[grid](...)` launch of `_fwd`, causal_conv1d.py:446-471,
 * together with `_fwd`'s T == 0 case (:437-444: final_states = initial_states, or zero).
 *   x               (B, T, D) at strides (stride_x_batch, stride_x_time, 1), type x_dtype
 *   weight          (D, W), type weight_dtype;   bias (D) or NULL, type bias_dtype
 *   initial_states  (B, W-1, D) or NULL, type init_dtype
 *   seq_idx         (B, T) int32 or NULL
 *   out             (B, T, D) contiguous, type x_dtype
 *   final_states    (B, W-1, D) contiguous or NULL: the last W-1 rows of concat(initial_states, x)
 *   silu            0 = no activation, 1 = SiLU
 */
int cc1d_fwd(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight,
             const void* bias, const void* initial_states, const int32_t* seq_idx, void* out,
             void* final_states, int64_t batch, int64_t seqlen, int64_t dim, int64_t width,
             int x_dtype, int weight_dtype, int bias_dtype, int init_dtype, int silu,
             void* stream);

/*
 * seq_idx for a packed variable-length batch, from cumulative sequence boundaries. The reference
 * takes seq_idx directly (causal_conv1d.py:594-596) and leaves building it to the caller; this
 * builds it on the device:
 *   cu_seqlens   (B, n_seqs + 1) int32, row b non-decreasing from 0: its sequences are
 *                [cu[b][i], cu[b][i+1])
 *   seq_idx      (B, T) int32 out: the sequence id (0 .. n_seqs-1) of each position, -1 (padding)
 *                at or past cu[b][n_seqs]
 */
int cc1d_seq_idx_from_cu_seqlens(const int32_t* cu_seqlens, int64_t n_seqs, int32_t* seq_idx,
                                 int64_t batch, int64_t seqlen, void* stream);

/*
 * Decode-time update of the streaming state. No counterpart kernel in the reference, which only
 * documents the state (`initial_states`/`final_states`, causal_conv1d.py:597-599); this applies L
 * new rows per batch row without a full forward:
 *   x               (B, L, D) at strides (stride_x_batch, stride_x_time, 1), type x_dtype
 *   conv_state      (n_slots, W-1, D) contiguous, type state_dtype, updated in place to the last
 *                   W-1 rows of concat(conv_state, x) (the final_states of the same forward)
 *   state_indices   (B) int32 slot of each batch row in conv_state, or NULL for slot b; a negative
 *                   slot skips the row (its output is left unwritten)
 *   out             (B, L, D) contiguous, type x_dtype: the forward's output for these rows,
 *                   computed with the same operations as cc1d_fwd
 */
int cc1d_update(const void* x, int64_t stride_x_batch, int64_t stride_x_time, void* conv_state,
                const int32_t* state_indices, const void* weight, const void* bias, void* out,
                int64_t batch, int64_t seqlen, int64_t dim, int64_t width, int x_dtype,
                int state_dtype, int weight_dtype, int bias_dtype, int silu, void* stream);

/*
 * Size in bytes of the fp32 workspace cc1d_bwd needs for its per-CTA weight/bias partial sums
 * (the `partials` buffer that `_bwd` allocates, causal_conv1d.py:493). Depends on the sizes, the
 * element type, the strides and 16-byte alignment of x and dout, and the current device.
 */
int64_t cc1d_bwd_workspace_bytes(const void* x, int64_t stride_x_batch, int64_t stride_x_time,
                                 const void* dout, int64_t stride_dout_batch,
                                 int64_t stride_dout_time, int64_t batch, int64_t seqlen,
                                 int64_t dim, int64_t width, int x_dtype);

/*
 * Backward. Replaces the `_bwd_kernel` and `_reduce_partials_kernel` launches of `_bwd`,
 * causal_conv1d.py:491-540, and `_bwd`'s T == 0 case (:480-489).
 *   dout            (B, T, D) at strides (stride_dout_batch, stride_dout_time, 1), type x_dtype
 *   dfinal_states   (B, W-1, D) or NULL, type x_dtype
 *   dx              (B, T, D) contiguous, type x_dtype
 *   dinit           (B, W-1, D) or NULL (requires initial_states), type init_dtype
 *   dweight, dbias  written in weight_dtype / bias_dtype (dbias only when bias is given) ...
 *   grad_f32        ... unless grad_f32 is non-NULL: then the fp32 vector
 *                   [dweight (D, W) row-major, dbias (D)] of D*(W+1) floats is written there
 *                   instead (dbias part zero without bias), ready for a cross-GPU all-reduce.
 *   workspace       device buffer of at least cc1d_bwd_workspace_bytes(...) bytes.
 * The weight/bias gradients are deterministic: a fixed-order sum of per-CTA partials.
 */
int cc1d_bwd(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight,
             const void* bias, const void* initial_states, const int32_t* seq_idx,
             const void* dout, int64_t stride_dout_batch, int64_t stride_dout_time,
             const void* dfinal_states, void* dx, void* dweight, void* dbias, void* dinit,
             float* grad_f32, void* workspace, int64_t workspace_bytes, int64_t batch,
             int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype,
             int bias_dtype, int init_dtype, int silu, void* stream);

/*
 * Backward without any device allocation, for callers that cannot allocate: runtimes that own all
 * of device memory in a pre-planned arena and must not call cudaMalloc after start-up, paths where
 * cudaMalloc/cudaFree could synchronise the device, and FFI callers with no device allocator. No
 * counterpart in the reference (its `_bwd` allocates the partials with torch, causal_conv1d.py:493).
 * Same arguments and results as cc1d_bwd, minus the workspace: the partial sums go to one fixed
 * 8 MiB array in the library's device memory (per GPU that loads the library, held until the
 * process exits). Problems whose cc1d_bwd_workspace_bytes() exceeds 8 MiB are rejected with
 * CC1D_ERR_SCRATCH_LIMIT before any device work. All calls on a device share the array, so calls
 * that overlap on the GPU race; order them on one stream. Nothing in the array must start at zero.
 * The first call on each device looks up the array's address (cudaGetSymbolAddress) with that
 * device current; make it before any stream capture. The address is kept until the process exits,
 * so cudaDeviceReset of a device after its first call is not supported. Error codes are those
 * cc1d_bwd returns for the same arguments, plus CC1D_ERR_SCRATCH_LIMIT.
 */
int cc1d_bwd_noalloc(const void* x, int64_t stride_x_batch, int64_t stride_x_time,
                     const void* weight, const void* bias, const void* initial_states,
                     const int32_t* seq_idx, const void* dout, int64_t stride_dout_batch,
                     int64_t stride_dout_time, const void* dfinal_states, void* dx,
                     void* dweight, void* dbias, void* dinit, float* grad_f32, int64_t batch,
                     int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype,
                     int bias_dtype, int init_dtype, int silu, void* stream);

/* One channel range of dout held in its own tensor (cc1d_bwd_split). Element (b, t, c) of the
 * piece, c in [0, channels), is at ptr + b*stride_batch + t*stride_time + c elements. */
typedef struct cc1d_dout_piece {
  const void* ptr;
  int64_t stride_batch;
  int64_t stride_time;
  int64_t channels;
} cc1d_dout_piece;

enum { CC1D_MAX_DOUT_PIECES = 4 };

/*
 * Backward with dout given as channel pieces and dx written through strides: the layout of a
 * Mamba-2 block, where the conv input xBC is a channel slice of the in_proj output zxbcdt and the
 * conv output is split into the SSM's x, B and C. The gradients of x, B and C arrive as separate
 * tensors; here they are read in place (no concatenation into one dout), and dx is written straight
 * into the xBC slice of the caller's d(zxbcdt) buffer (no second concatenation). No counterpart in
 * the reference, which takes one dout and returns a fresh dx (causal_conv1d.py:475-541).
 *   dout_pieces     n_pieces (1..CC1D_MAX_DOUT_PIECES) pieces, covering channels [0, dim) in order;
 *                   every piece boundary a multiple of 128 channels (64 for fp32)
 *   dx              (B, T, D) at strides (stride_dx_batch, stride_dx_time, 1)
 * Everything else as cc1d_bwd; size the workspace with cc1d_bwd_workspace_bytes() given the first
 * piece as dout. The call needs the TMA path: widths 2..16; x, every piece and dx 16-byte aligned
 * with 16-byte-multiple batch/time strides. Otherwise it returns CC1D_ERR_LAYOUT before any device
 * work, and the caller concatenates dout and calls cc1d_bwd. Graph-capturable like cc1d_bwd.
 */
int cc1d_bwd_split(const void* x, int64_t stride_x_batch, int64_t stride_x_time,
                   const void* weight, const void* bias, const void* initial_states,
                   const int32_t* seq_idx, const cc1d_dout_piece* dout_pieces, int n_pieces,
                   const void* dfinal_states, void* dx, int64_t stride_dx_batch,
                   int64_t stride_dx_time, void* dweight, void* dbias, void* dinit,
                   float* grad_f32, void* workspace, int64_t workspace_bytes, int64_t batch,
                   int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype,
                   int bias_dtype, int init_dtype, int silu, void* stream);

/*
 * Copies a (batch, seqlen, channels) block of elem_bytes-sized elements from src to dst, each at its
 * own batch/time strides (in elements; channel stride 1). The glue around cc1d_bwd_split: it places
 * dz and ddt in d(zxbcdt) at full bandwidth (16-byte vectors when the addresses and strides allow),
 * where an element-wise copy into a strided slice runs at a fraction of it. No counterpart in the
 * reference. Graph-capturable; allocates nothing.
 */
int cc1d_copy_channels(void* dst, int64_t dst_stride_batch, int64_t dst_stride_time,
                       const void* src, int64_t src_stride_batch, int64_t src_stride_time,
                       int64_t batch, int64_t seqlen, int64_t channels, int elem_bytes,
                       void* stream);

/*
 * Reads the device status word of the current device after synchronising it, and clears it when
 * `clear` is non-zero. Bit 0 set: a kernel gave up waiting on one of its pipeline barriers
 * (bounded at one second) and returned early, so its outputs are incomplete. The word's device
 * address is looked up once per device and kept, so cudaDeviceReset after the library's first
 * call on a device is not supported.
 */
int cc1d_status(uint32_t* status, int clear);

/*
 * Self-test of the failure detection: launches one block whose threads wait on a shared-memory
 * mbarrier that nothing ever completes, with the same bounded wait as the kernels (about one
 * second), so the wait gives up, sets bit 0 of the device status word and the kernel returns; no
 * fault, and the context stays usable. cc1d_status() then reports the bit. No counterpart in the
 * reference (its Triton kernels have no waits); it exists so that the timeout path can be checked
 * on a real GPU.
 */
int cc1d_selftest_wait_timeout(void* stream);

/* Human-readable text for a CC1D_ERR_* code. */
const char* cc1d_error_string(int code);

/* The cudaError_t of the last failed CUDA call made by this library on the calling thread. */
int cc1d_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* CAUSAL_CONV1D_B200_H_ */
