/*
 * trring.h -- C ABI of the B200 (sm_100a) three-core tensor-ring linear operator.
 *
 *   y[t,(p,q,r)] = sum_{i,j,k,a,b,c} x[t,(i,j,k)] A[a,p,i,b] B[b,q,j,c] C[c,r,k,a]
 *
 * Cores use the reference's storage order [rank, output_mode, input_mode, rank]
 * (factorized_inference/reference.py:17-21, 66-73); x is [tokens, i*j*k] row-major with the
 * first input mode slowest, y is [tokens, p*q*r] with the first output mode slowest
 * (reference.py:119,125).  The dense weight is never formed.
 *
 * Every entry point returns an int status (TR_OK == 0, negative on error); no C++ exception
 * crosses this boundary.  The library never allocates device memory: packed cores and the
 * workspace are buffers the caller owns, sized by tr_packed_bytes / tr_workspace_bytes.
 * Device pointers are plain pointers on the plan's device; `stream` is a cudaStream_t
 * (NULL = legacy default stream).
 *
 * Reference interfaces these replace (paths inside danila-permogorskii/kernel-task):
 *   tr_plan_create + tr_pack_cores   <- PreparedTRKernel.__init__ and pack_cores
 *                                       (src/factorized_inference/tr_kernel.py:190-228, 86-99)
 *   tr_forward                       <- PreparedTRKernel.__call__ (tr_kernel.py:264-319) and
 *                                       the extension entry points tr_ring_forward /
 *                                       tr_ring_forward_v3 / tr_ring_forward_v3t
 *                                       (src/factorized_inference/csrc/tr_ring.cu:448-463,
 *                                       1108-1141, 1156-1192)
 *   tr_workspace_bytes               <- the design-B workspace sizing in PreparedTRKernel.__call__
 *                                       (tr_kernel.py:290-296, 314-317)
 *   tr_plan_destroy                  <- releasing the PreparedTRKernel (Python GC in the reference)
 *   tr_forward_epilogue              <- PreparedTRKernel.accumulate (tr_kernel.py:230-243) and
 *                                       the extension's forward_fp32 (csrc/v3g/bind.cu:84-91),
 *                                       with the consumers below fused into the same launch
 *   tr_consume_silu_mul              <- consume_silu_mul (csrc/v3g/bind.cu:93-108, 123-133)
 *   tr_consume_add                   <- consume_add (csrc/v3g/bind.cu:110-121, 135-148)
 */
#ifndef TRRING_H
#define TRRING_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference raises ValueError for shape errors (reference.py:27-31,85-96)
 * and RuntimeError through TORCH_CHECK (tr_ring.cu:416-418,453-457); the torch binding maps
 * TR_ERR_INVALID to ValueError and everything else to RuntimeError. */
enum tr_status {
  TR_OK = 0,
  TR_ERR_INVALID = -1,     /* bad argument: shape, null pointer, unknown dtype, negative T   */
  TR_ERR_UNSUPPORTED = -2, /* valid spec, but no kernel of this build handles it           */
  TR_ERR_WORKSPACE = -3,   /* workspace pointer missing or smaller than tr_workspace_bytes */
  TR_ERR_CUDA = -4,        /* a CUDA runtime call failed (message: tr_last_error)          */
  TR_ERR_ALIGN = -5,       /* a pointer is not aligned as required (16 bytes)              */
  TR_ERR_TIMEOUT = -6      /* a bounded device-side wait gave up (status word set)         */
};

/* Element types of cores, x and y (one type per plan). */
enum tr_dtype { TR_F32 = 0, TR_F16 = 1, TR_BF16 = 2 };

/* Shape of one operator.  Mirrors TRSpec (reference.py:15-50): one rank for all three ring
 * links; core k has shape [rank, output_modes[k], input_modes[k], rank]. */
typedef struct tr_spec {
  int32_t input_modes[3];
  int32_t output_modes[3];
  int32_t rank;
} tr_spec;

/* Per-call kernel geometry override (tests and tuning).  Zero fields mean "planner's choice".
 *   tokens_per_tile : tokens per CTA row tile
 *   cluster         : CTAs per thread-block cluster that split a tile's ring pieces and add
 *                     their partial sums (through DSMEM in the decode kernel, through
 *                     per-CTA workspace areas in L2 in the tcgen05 kernels)
 *   clusters        : clusters per row tile (>1 adds the workspace slot reduction)
 *   kernel          : 0 auto, 1 generic CUDA-core kernel, 2 mma.sync fused tile kernel,
 *                     3 tcgen05 fused kernel (ring rank padded to 8 or 16),
 *                     4 mma.sync decode kernel (T*o1 and T*i2 <= 32; here `cluster` splits
 *                     the pieces and `clusters` the output modes),
 *                     5 tcgen05 slab kernel (the ring rank cut into slabs of 8; ranks up
 *                     to 32)                                                               */
typedef struct tr_tiling {
  int32_t tokens_per_tile;
  int32_t cluster;
  int32_t clusters;
  int32_t kernel;
} tr_tiling;

typedef struct tr_plan tr_plan;

/* Validate the spec, pick the contraction order (the cheapest of the six ring orders, no
 * dense W), and lay out the packed cores.  Host only; no device memory is touched.
 * `device` is the CUDA ordinal every later call must use.                                     */
int tr_plan_create(const tr_spec* spec, int32_t dtype, int32_t device, tr_plan** out);
void tr_plan_destroy(tr_plan* plan);

/* Bytes of the packed-core buffer (16-byte aligned device memory, caller-owned). */
int tr_packed_bytes(const tr_plan* plan, size_t* bytes);

/* Pack the three caller cores (contiguous device tensors of the plan's dtype, shapes
 * [R,o_k,i_k,R]) into `packed`.  Cores are read, never written.  Stream-ordered.
 * The forward kernels may start their first reads of `packed` while the previous kernel of the
 * stream is still running (programmatic dependent launch); write a packed buffer only through
 * this call (it ends with a normally serialized launch), or with a stream-ordered copy.      */
int tr_pack_cores(const tr_plan* plan, const void* const cores[3], void* packed, void* stream);

/* Workspace bytes tr_forward needs for `tokens` rows (0 when the chosen kernel needs none).
 * A workspace must be zero-filled once before its first use (tr_workspace_clear); every
 * forward leaves it ready for the next call.  One workspace serves one stream at a time.      */
int tr_workspace_bytes(const tr_plan* plan, int64_t tokens, size_t* bytes);
/* Workspace bytes for an explicit geometry (see tr_forward_tiled; NULL = planner's choice). */
int tr_workspace_bytes_tiled(const tr_plan* plan, int64_t tokens, const struct tr_tiling* tiling,
                             size_t* bytes);
int tr_workspace_clear(void* workspace, size_t bytes, void* stream);

/* Device status of the calls that used `workspace`: TR_OK, or TR_ERR_TIMEOUT when a bounded
 * wait inside a tcgen05 kernel gave up (its y is then not valid).  The kernels record a timeout
 * in the first workspace word instead of hanging; a forward call returns before its kernel
 * runs, so only this read (stream-ordered: it synchronises `stream`) can see it.  `reset` != 0
 * clears the word, which every later call otherwise finds set.  A zero-byte workspace has no
 * status (the decode and mma kernels have no waits that can expire).  The reference has no
 * counterpart: its design-B kernels have no bounded waits (csrc/tr_ring.cu:302-337).        */
int tr_workspace_status(void* workspace, size_t workspace_bytes, int32_t* status, int32_t reset,
                        void* stream);

/* Polls a bounded device-side wait of this plan's tcgen05 kernels makes before it gives up and
 * reports TR_ERR_TIMEOUT (0 = built-in limit, about a second).  For tests of the timeout path:
 * a tiny limit makes the waits expire on a healthy GPU.  No reference counterpart.            */
int tr_plan_set_wait_limit(tr_plan* plan, uint32_t polls);

/* y[tokens, d_out] = TR(x[tokens, d_in]).  x, y: contiguous row-major, plan dtype, 16-byte
 * aligned.  tokens == 0 is a no-op.  Launches exactly one kernel on `stream`.                 */
int tr_forward(const tr_plan* plan, const void* packed, const void* x, int64_t tokens, void* y,
               void* workspace, size_t workspace_bytes, void* stream);

/* tr_forward on host buffers: x_host [tokens, d_in] is copied into the device staging buffer
 * x_dev, the forward writes y_dev, and y_dev is copied into y_host [tokens, d_out], as three
 * stream-ordered operations (two cudaMemcpyAsync and one kernel) issued by one call.  The call
 * returns before they finish: synchronise `stream` before reading y_host.  Page-locked host
 * memory keeps the copies asynchronous.  x_dev and y_dev are caller-owned device buffers of at
 * least tokens * d_in and tokens * d_out elements, 16-byte aligned; they may be reused by the
 * next call on the same stream.  For hosts whose data lives in host memory (a plugin, another
 * language's FFI); the reference's callers always pass device tensors, so it has no
 * counterpart there.                                                                          */
int tr_forward_host(const tr_plan* plan, const void* packed, const void* x_host, int64_t tokens,
                    void* y_host, void* x_dev, void* y_dev, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Same as tr_forward with an explicit geometry (NULL = planner's choice). */
int tr_forward_tiled(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                     void* y, void* workspace, size_t workspace_bytes, const tr_tiling* tiling,
                     void* stream);

/* tr_forward without a caller workspace, for callers that cannot allocate device memory:
 * for example a plugin or foreign-language host that has no CUDA allocator of its own, or a
 * serving loop that must not call cudaMalloc (it can synchronise the device) once running.
 * It has no counterpart in the reference, whose callers always own a torch allocator.
 *
 * The scratch it needs lives in a fixed 8 MiB array inside this library (TR_NOALLOC_SCRATCH_
 * BYTES), which every GPU that loads the library holds until the process exits.  A call whose
 * token count needs more returns TR_ERR_WORKSPACE; use tr_forward with a workspace instead.
 * The call allocates nothing: no cudaMalloc, cudaFree or allocating library routine.  Its first
 * call on a device looks up the array's device address on that device; make that first call
 * before any stream capture.  All calls share the one array and it keeps the last call's
 * contents, so calls whose kernels overlap on the GPU (two streams, two threads) race and give
 * wrong results; issue them in one stream order.  fp16/bf16 plans only.
 * The array's device address is looked up once per device and kept for the life of the
 * process: after cudaDeviceReset, or after the device's primary context is released and
 * created again, that address is stale, so do not call this entry point after either.
 * Each call issues two operations on `stream`: a cudaMemsetAsync that zeroes the array's
 * arrival counters (a guard against an earlier call whose kernel never ran to its end), then
 * the kernel.                                                                                */
#define TR_NOALLOC_SCRATCH_BYTES (8u << 20)
int tr_forward_noalloc(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                       void* y, void* stream);

/* Epilogues applied to each finished y element v inside the forward kernel, before the one
 * store of y (no extra launch, no fp32 round trip through memory):
 *   TR_EPI_NONE      y = v
 *   TR_EPI_ADD       y = aux + v            (residual add after a projection)
 *   TR_EPI_SILU_MUL  y = silu(aux) * v      (gated MLP: aux = gate(x), v = up(x))
 * aux is [tokens, d_out] row-major, fp32 or the plan's dtype, 16-byte aligned; it may be y
 * itself (an in-place residual add) but must not overlap y otherwise, nor x.  out_dtype is
 * TR_F32 (y stored as fp32: the reference's accumulate / forward_fp32) or the plan's dtype.
 * The arithmetic is fp32: v + aux, and aux / (1 + exp(-aux)) * v, rounded once on store.   */
enum tr_epilogue_kind { TR_EPI_NONE = 0, TR_EPI_ADD = 1, TR_EPI_SILU_MUL = 2 };
typedef struct tr_epilogue {
  int32_t kind;      /* tr_epilogue_kind                          */
  int32_t out_dtype; /* TR_F32 or the plan's dtype                */
  const void* aux;   /* second operand (unused for TR_EPI_NONE)   */
  int32_t aux_dtype; /* TR_F32 or the plan's dtype                */
} tr_epilogue;

/* tr_forward_tiled with an epilogue (NULL epilogue = plain forward in the plan's dtype). */
int tr_forward_epilogue(const tr_plan* plan, const void* packed, const void* x, int64_t tokens,
                        void* y, const tr_epilogue* epilogue, void* workspace,
                        size_t workspace_bytes, const tr_tiling* tiling, void* stream);

/* The reference's stand-alone consumers of fp32 forward outputs, for callers that keep the
 * unfused order.  n elements, n % 4 == 0, all pointers 16-byte aligned, out_dtype TR_F16 or
 * TR_BF16.  Like the reference, each clears (zero-fills) the fp32 inputs it consumed.
 *   tr_consume_silu_mul: out = silu(g) * u;  g, u fp32, both cleared
 *   tr_consume_add:      out = h + y;        h in out_dtype, y fp32, y cleared             */
int tr_consume_silu_mul(float* g, float* u, void* out, int32_t out_dtype, int64_t n,
                        void* stream);
int tr_consume_add(const void* h, float* y, void* out, int32_t out_dtype, int64_t n,
                   void* stream);

/* The geometry tr_forward would use for `tokens` (after clamping to this device). */
int tr_plan_tiling(const tr_plan* plan, int64_t tokens, tr_tiling* out);

/* JSON description of the plan (order, canonical modes, packed layout, per-path FLOPs). */
int tr_plan_describe(const tr_plan* plan, char* buf, size_t len);

/* Algorithmic FLOPs per token of the chosen contraction order (2 * MACs). */
int tr_plan_flops_per_token(const tr_plan* plan, double* flops);

const char* tr_status_string(int status);
/* Last error message of the calling thread (CUDA error text or argument diagnostics). */
const char* tr_last_error(void);

/* An empty kernel on `stream`: the launch floor the roofline is bounded by. */
int tr_empty_launch(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRRING_H */
