/*
 * cfk.h -- C ABI of the B200 (sm_100a) Evoformer kernels.
 *
 * This is the drop-in boundary beneath the XLA FFI handlers.  Every entry point takes raw
 * device pointers, sizes, a dtype code and a CUDA stream; it validates its arguments, enqueues
 * its kernels on that stream and returns.  No entry point synchronises, allocates device memory
 * or creates streams, so every call can be recorded into a CUDA graph (XLA's command buffers).
 * Scratch memory, where a kernel needs some, is passed in by the caller; its size comes from the
 * matching *_workspace_size() query.
 *
 * Return value: CFK_OK (0) or one of the cfk_status codes; cfk_last_error() then gives a
 * message for the failing call on the calling thread.
 *
 * Citations name the reference interface each entry point replaces
 * (sokrypton/colabfold-legacy-kernels, path:line).
 */
#ifndef CFK_H_
#define CFK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CFK_API __attribute__((visibility("default")))
#else
#define CFK_API
#endif

/* A cudaStream_t; declared without the CUDA headers so this file stays plain C. */
typedef struct CUstream_st* cfk_stream_t;

/* Element type of the 16-bit tensors (q/k/v/out, x/y, weights).  The reference is F16 only. */
typedef enum {
    CFK_F16 = 0,
    CFK_BF16 = 1,
} cfk_dtype;

typedef enum {
    CFK_OK = 0,
    CFK_ERR_INVALID_ARGUMENT = 1, /* bad shape, dtype, alignment or workspace size */
    CFK_ERR_UNSUPPORTED_DEVICE = 2, /* the current device is not compute capability 10.0 */
    CFK_ERR_LAUNCH = 3,             /* a CUDA launch or attribute call failed */
} cfk_status;

/* Message of the last failing call on this thread ("" if none). */
CFK_API const char* cfk_last_error(void);

/* Library version string. */
CFK_API const char* cfk_version(void);

/* ------------------------------------------------------------------------------------------ */
/* Attention with an additive pair bias and a key mask.                                       */
/*                                                                                            */
/*   logit[n,h,i,j] = scale * <q[n,h,i,:], k[n,h,j,:]> + bias[h,i,j]   if kmask[n,j] != 0     */
/*                  = -1e4                                             otherwise (replaced,   */
/*                                                                     bias dropped)          */
/*   out[n,h,i,:]   = sum_j softmax_j(logit[n,h,i,:]) * v[n,h,j,:]                            */
/*                                                                                            */
/* Layouts (row-major, contiguous): q,out [N,H,Sq,D]; k,v [N,H,Sk,D]; bias [H,Sq,Sk] shared   */
/* by all n; kmask u8 [N,Sk].  D in {8,16,32,64}.  fp32 accumulation and softmax.             */
/* ------------------------------------------------------------------------------------------ */

/* Forward.  Replaces VoltaMma / VoltaWmma (cuda/volta_mma_attn.cu:304-351,
 * cuda/volta_wmma_attn.cu:264-311).  lse may be NULL; otherwise it receives the natural-log
 * log-sum-exp of each row, f32 [N,H,Sq], which the backward needs. */
CFK_API int cfk_attn_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, void* out, float* lse,
                 int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale);

/* Bytes of scratch memory cfk_attn_bwd needs for these sizes. */
CFK_API int cfk_attn_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                size_t* bytes);

/* Backward (no counterpart in the reference, which is forward-only; it is the autodiff of
 * cuda/volta_mma_attn.cu:139-271).  Inputs are the forward's inputs plus out, its lse and dout.
 * Outputs: dq [N,H,Sq,D], dk, dv [N,H,Sk,D] in dtype; dbias f32 [H,Sq,Sk] = sum over n of
 * dlogit (zero where masked).  Masked logits are constants, so they pass no gradient. */
CFK_API int cfk_attn_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* q, const void* k,
                 const void* v, const void* bias, const uint8_t* kmask, const void* out,
                 const float* lse, const void* dout, void* dq, void* dk, void* dv, float* dbias,
                 void* workspace, size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq,
                 int64_t Sk, int64_t D, float scale);

/* The three stages of cfk_attn_bwd, callable one by one with the same arguments (no
 * counterpart in the reference): phase 0 computes the row statistics (delta =
 * rowsum(dout * out), with lse) and, for D <= 32, zeroes dq, dk, dv, into which phase 1 adds
 * its partial sums; phase 1 is the main tcgen05 kernel (it completes dbias, and for D <= 32
 * dq, dk, dv); phase 2 converts D = 64's f32 accumulators to dtype (nothing for D <= 32).
 * Issued in order on one stream they equal cfk_attn_bwd; a caller may, for example, start a
 * collective on dbias after phase 1 while phase 2 runs. */
CFK_API int cfk_attn_bwd_phase(int phase, cfk_stream_t stream, cfk_dtype dtype, const void* q,
                       const void* k, const void* v, const void* bias, const uint8_t* kmask,
                       const void* out, const float* lse, const void* dout, void* dq, void* dk,
                       void* dv, float* dbias, void* workspace, size_t workspace_bytes,
                       int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale);

/* Strided ("view") forms of the three calls above (no counterpart in the reference).  Each
 * [N,H,S,D] tensor is described by a cfk_view: the element strides of its batch, head and
 * sequence axes, the D axis staying contiguous.  Attention over the other residue axis
 * (triangle attention around the ending node, MSA column attention) or over a [N,S,H,D]
 * layout then needs no transposed copy: the kernels' TMA descriptors and row addressing take
 * the strides.  Strides of axes longer than 1 must be positive multiples of 8 elements; views
 * NULL means packed, as above.  Output views must not overlap each other or the inputs.
 * bias, kmask, lse, dbias and the workspace stay packed. */
typedef struct cfk_view {
    int64_t b, h, s;
} cfk_view;

/* views[0..3]: q, k, v, out */
CFK_API int cfk_attn_fwd_strided(cfk_stream_t stream, cfk_dtype dtype, const void* q,
                         const void* k, const void* v, const void* bias, const uint8_t* kmask,
                         void* out, float* lse, int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                         int64_t D, float scale, const cfk_view* views);

/* views[0..7]: q, k, v, out, dout, dq, dk, dv */
CFK_API int cfk_attn_bwd_strided(cfk_stream_t stream, cfk_dtype dtype, const void* q,
                         const void* k, const void* v, const void* bias, const uint8_t* kmask,
                         const void* out, const float* lse, const void* dout, void* dq, void* dk,
                         void* dv, float* dbias, void* workspace, size_t workspace_bytes,
                         int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale,
                         const cfk_view* views);
CFK_API int cfk_attn_bwd_phase_strided(int phase, cfk_stream_t stream, cfk_dtype dtype,
                               const void* q, const void* k, const void* v, const void* bias,
                               const uint8_t* kmask, const void* out, const float* lse,
                               const void* dout, void* dq, void* dk, void* dv, float* dbias,
                               void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                               int64_t Sq, int64_t Sk, int64_t D, float scale,
                               const cfk_view* views);

/* The sigmoid gate of the Evoformer's attention modules, fused (no counterpart in the
 * reference, whose caller runs it in jnp): forward y = sigmoid(g) * o; backward
 * d_o = dy * sigmoid(g), dg = dy * o * sigmoid(g) * (1 - sigmoid(g)).  n elements of dtype
 * each, every buffer 16-byte aligned; f32 arithmetic, each output rounded once. */
CFK_API int cfk_gate_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* g, const void* o,
                 void* y, int64_t n);
CFK_API int cfk_gate_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* g, const void* o,
                 const void* dy, void* d_o, void* dg, int64_t n);

/* ------------------------------------------------------------------------------------------ */
/* LayerNorm over the last axis: y = (x - mean) * rstd * gamma + beta,                        */
/* rstd = 1/sqrt(var + eps).  x, y [M,C] in dtype; gamma, beta f32 [C]; statistics in f32.    */
/* ------------------------------------------------------------------------------------------ */

/* Forward.  Replaces VoltaLayerNorm (cuda/volta_ops.cu:62-95).  mean and rstd (f32 [M]) may be
 * NULL; when given they receive the row statistics for the backward. */
CFK_API int cfk_ln_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const float* gamma,
               const float* beta, void* y, float* mean, float* rstd, int64_t M, int64_t C,
               float eps);

/* Bytes of scratch memory cfk_ln_bwd needs. */
CFK_API int cfk_ln_bwd_workspace_size(int64_t M, int64_t C, size_t* bytes);

/* Backward (no counterpart in the reference; autodiff of cuda/volta_ops.cu:40-58).
 * mean/rstd may be NULL, in which case they are recomputed from x.  Outputs dx [M,C] in dtype,
 * dgamma, dbeta f32 [C] (written, not accumulated). */
CFK_API int cfk_ln_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const float* gamma,
               const float* mean, const float* rstd, const void* dy, void* dx, float* dgamma,
               float* dbeta, void* workspace, size_t workspace_bytes, int64_t M, int64_t C,
               float eps);

/* LayerNorm backward that allocates nothing and takes no workspace.  It has no counterpart in
 * the reference.  It is for callers that cannot provide device memory: an XLA FFI handler gets
 * only the buffers its binding declares and must not allocate, so a handler with the
 * reference's buffer list (no workspace result) cannot feed cfk_ln_bwd; hosts that plan every
 * device allocation up front are in the same position.  The per-CTA dgamma/dbeta partials live
 * in a static device array of 2.5 MiB (held by every GPU that loads the library until the
 * process exits), so C must be <= 1024 (larger C is rejected with CFK_ERR_INVALID_ARGUMENT).
 * The first call on a device looks up the array's device address with that device current;
 * make that first call before any stream capture (a lookup that fails is not cached: the next
 * call retries it).  Device ordinals 0-63 are served.  All calls share the array: each launch
 * rewrites the partials it reads, so nothing carries over, but calls that overlap on the GPU
 * (for example on two streams of one device) race.  Results equal cfk_ln_bwd's up to the
 * summation order of dgamma and dbeta. */
CFK_API int cfk_ln_bwd_noalloc(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                       const float* gamma, const float* mean, const float* rstd, const void* dy,
                       void* dx, float* dgamma, float* dbeta, int64_t M, int64_t C, float eps);

/* ------------------------------------------------------------------------------------------ */
/* Gated dual projection:                                                                     */
/*   out[m,n] = mask[m] * (x@wp + bp)[m,n] * sigmoid((x@wg + bg)[m,n])                        */
/* x [M,K], wp, wg [K,N] row-major, bp, bg [N], mask [M], out [M,N]; all in dtype.            */
/* ------------------------------------------------------------------------------------------ */

/* Forward.  Replaces VoltaGdp / VoltaGdpWmma (cuda/volta_ops.cu:210-265,
 * cuda/volta_gdp_wmma.cu:99-140).  N must be a multiple of 8, as in the reference. */
CFK_API int cfk_gdp_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* wp,
                const void* bp, const void* wg, const void* bg, const void* mask, void* out,
                int64_t M, int64_t K, int64_t N);

/* LayerNorm fused into the forward (no counterpart in the reference; the two-step
 * x = LayerNorm(z) (cuda/volta_ops.cu:28-60) then VoltaGdp of triangle multiplication):
 * out = gdp(LayerNorm(z; gamma, beta, eps)) without writing x to memory.  z [M,K] in dtype,
 * gamma, beta f32 [K]; mean, rstd (f32 [M]) may be NULL.  Shapes outside the tcgen05 path
 * (cfk_ln_gdp_fwd_workspace_size reports a nonzero size for them) stage x in the workspace. */
CFK_API int cfk_ln_gdp_fwd_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes);
CFK_API int cfk_ln_gdp_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* z, const float* gamma,
                   const float* beta, float eps, const void* wp, const void* bp,
                   const void* wg, const void* bg, const void* mask, void* out, float* mean,
                   float* rstd, void* workspace, size_t workspace_bytes, int64_t M, int64_t K,
                   int64_t N);

/* Bytes of scratch memory cfk_gdp_bwd needs. */
CFK_API int cfk_gdp_bwd_workspace_size(int64_t M, int64_t K, int64_t N, size_t* bytes);

/* Backward (no counterpart in the reference; autodiff of cuda/volta_ops.cu:185-207 with mask
 * treated as a constant).  Outputs dx [M,K] in dtype; dwp, dwg f32 [K,N]; dbp, dbg f32 [N]. */
CFK_API int cfk_gdp_bwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* wp,
                const void* bp, const void* wg, const void* bg, const void* mask,
                const void* dout, void* dx, float* dwp, float* dbp, float* dwg, float* dbg,
                void* workspace, size_t workspace_bytes, int64_t M, int64_t K, int64_t N);

/* ------------------------------------------------------------------------------------------ */
/* Plain projections of the attention modules (no counterpart in the reference: the modules  */
/* that call its kernels do these GEMMs in the host framework).  The forward is the tiling   */
/* of cuda/volta_ops.cu:143-207 without the gate.                                             */
/* ------------------------------------------------------------------------------------------ */

/* y = x w + b: x [M,K], w [K,N] row-major, b [N] or NULL, all in dtype, f32 accumulation.
 * Columns [0, n_split) go to y0 (row stride ld0 elements), columns [n_split, N) to y1 (row
 * stride ld1; unused when n_split = N), so one call can fill two buffers.  n_split is N or a
 * multiple of 128 in (0, N).  N % 8 == 0. */
CFK_API int cfk_linear_fwd(cfk_stream_t stream, cfk_dtype dtype, const void* x, const void* w,
                   const void* b, void* y0, int64_t ld0, void* y1, int64_t ld1,
                   int64_t n_split, int64_t M, int64_t K, int64_t N);

/* One column block of a projection's output gradient, for the backward calls below:
 * dy [M, n] in dtype with row stride ld elements, the block's weight w [K, n] (dtype,
 * row-major; cfk_linear_bwd_dx), and its f32 gradients dw [K, n] and db [n] (db may be NULL;
 * cfk_linear_bwd_dw).  n % 8 == 0. */
typedef struct cfk_linear_seg {
    const void* dy;
    int64_t ld;
    int64_t n;
    const void* w;
    float* dw;
    float* db;
} cfk_linear_seg;

#define CFK_LINEAR_MAX_SEGS 4

/* dx [M,K] (dtype) = sum over the n_segs (1..4) blocks of dy_s w_s^T, f32 accumulation. */
CFK_API int cfk_linear_bwd_dx(cfk_stream_t stream, cfk_dtype dtype, const cfk_linear_seg* segs,
                      int n_segs, void* dx, int64_t M, int64_t K);

/* Bytes of scratch memory cfk_linear_bwd_dw needs for these blocks on the current device. */
CFK_API int cfk_linear_bwd_dw_workspace_size(const cfk_linear_seg* segs, int n_segs, int64_t M,
                                     int64_t K, size_t* bytes);

/* dw_s = x^T dy_s and db_s = the column sums of dy_s (f32) for each block, x [M,K] in dtype
 * read once; deterministic (partial sums over row groups added in a fixed order). */
CFK_API int cfk_linear_bwd_dw(cfk_stream_t stream, cfk_dtype dtype, const void* x,
                      const cfk_linear_seg* segs, int n_segs, int64_t M, int64_t K,
                      void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------------------------------ */
/* dbias across GPUs over peer memory (no counterpart in the reference, which runs on one     */
/* device: cuda/volta_mma_attn.cu:295 parallelises over its grid only).                       */
/* ------------------------------------------------------------------------------------------ */

#define CFK_IPC_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer for dbias [H, Sq, Sk] f32: dbias itself (rounded up to
 * 256 bytes) followed by a 128-byte sync block.  0 for a size outside [1, 2^20] per axis. */
CFK_API size_t cfk_dbias_exchange_bytes(int64_t H, int64_t Sq, int64_t Sk);

/* Allocates `bytes` of device memory on the current device, zeroed, and returns it with its
 * CUDA IPC handle (CFK_IPC_HANDLE_BYTES bytes) for the other processes of the node.  The only
 * allocating entry points of the library are this one and cfk_ipc_open: call them at set-up,
 * outside stream capture (synchronous). */
CFK_API int cfk_ipc_alloc(size_t bytes, void** dptr, void* handle);

/* Maps another process's cfk_ipc_alloc buffer into this one (on the current device, with peer
 * access enabled); a process cannot open its own handle. */
CFK_API int cfk_ipc_open(const void* handle, void** dptr);

/* Unmaps a buffer mapped by cfk_ipc_open. */
CFK_API int cfk_ipc_close(void* dptr);

/* Frees a buffer from cfk_ipc_alloc (after every peer has unmapped it). */
CFK_API int cfk_ipc_free(void* dptr);

/* Reduce-scatter of dbias by query rows, for attention rows sharded across `world` GPUs (one
 * process each).  buffers: host array of `world` device pointers, rank r's exchange buffer
 * (cfk_dbias_exchange_bytes(H, Sq, Sk) bytes from cfk_ipc_alloc, peers' through cfk_ipc_open);
 * its first H*Sq*Sk floats hold rank r's partial dbias [H, Sq, Sk] (the dbias output of its
 * backward, complete before this call on `stream`).  Writes out [H, Sq/world, Sk] = the sum over
 * ranks, in rank order 0..world-1 (deterministic), of rows [rank*Sq/world, (rank+1)*Sq/world)
 * of every head.  One kernel reads those rows straight from the peers' buffers over NVLink;
 * every rank must make the same calls with the same shape in the same order.  When the launch
 * completes, no peer reads this rank's dbias any more, so it may be overwritten.  The call
 * number lives in the sync blocks (device memory), so the launch takes no per-call argument.
 * A wait for another rank gives up after the wait limit and sets 4 in the status word; the
 * buffers' counters then no longer agree across ranks: allocate new ones.  2 <= world <= 8,
 * Sq % world == 0, Sk % 4 == 0, out 16-byte aligned, buffers 256-byte aligned. */
CFK_API int cfk_dbias_reduce_scatter(cfk_stream_t stream, void* const* buffers, int world,
                                     int rank, int64_t H, int64_t Sq, int64_t Sk, float* out);

/* ------------------------------------------------------------------------------------------ */
/* Diagnostics (no counterpart in the reference).                                             */
/* ------------------------------------------------------------------------------------------ */

/* Every wait inside a kernel (on a barrier or on the tensor-memory pipeline) gives up after
 * the device's wait limit (one second unless cfk_set_wait_limit_ns changed it).  It then
 * records a code in a per-device status word and the kernel returns early instead of hanging;
 * the outputs of every launch that ran while the word was set are undefined.  This reads the
 * word of the current device (0 = no timeout seen; bit 1 = a barrier wait ran past its limit;
 * bit 4 = a wait for another GPU in cfk_dbias_reduce_scatter did). */
CFK_API int cfk_device_status(uint32_t* code);

/* Clears the status word of the current device. */
CFK_API int cfk_clear_device_status(void);

/* Sets the wait limit of the current device in nanoseconds, in [1e5, 6e11] (0.1 ms to ten
 * minutes); launches enqueued afterwards use it.  A shared GPU that time-slices between
 * processes can stretch a healthy wait, so a caller that shares its GPU may raise the limit.
 * Synchronous (a copy into device memory); call it outside stream capture. */
CFK_API int cfk_set_wait_limit_ns(uint64_t ns);

/* Reads the wait limit of the current device. */
CFK_API int cfk_get_wait_limit_ns(uint64_t* ns);

/* Self-test of the give-up path: launches one warp that waits on a barrier no thread arrives
 * on, through the kernels' own waiting loop, with a limit of limit_ns (in [1e5, 1e8]; 0 = the
 * device's limit).  The wait gives up, records 1 in the status word and the kernel returns;
 * *result (device memory, 4 bytes) is set to 1.  No TMA or tensor-core work is in flight, so
 * the context stays usable.  Clear the status word before the next real launch. */
CFK_API int cfk_test_wait_timeout(cfk_stream_t stream, uint64_t limit_ns, uint32_t* result);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CFK_H_ */
