/*
 * aria_q4.h -- C ABI of the B200 (sm_100a) Q4_0 projection library, libaria_q4.so.
 *
 * Drop-in boundary for lold3344/ARIA's quantised inference path.  The reference
 * binds its GPU work from Rust through cudarc: kernels by name from a PTX module
 * (src/transformer_cuda.rs:832-890) and cuBLAS through the `gemm()` helper
 * (src/transformer_cuda.rs:615-640).  These functions replace, for Q4_0
 * weights, the five projection GEMMs and the CPU packer.
 *
 * Conventions (all entry points):
 *   - every pointer is a device pointer unless stated otherwise; `stream` is a
 *     cudaStream_t (CUstream) passed as void*, NULL = legacy default stream;
 *   - calls are stream-ordered and asynchronous: no host synchronisation and
 *     no allocation.  Calls on distinct streams or threads share no buffers
 *     except two per-device objects: the device error code of the bounded
 *     waits (aria_q4_take_device_error: one per device, so a wait that expires
 *     in one stream is reported to whichever thread reads the code first) and
 *     the static scratch of aria_q4_0_matmul_static_ws;
 *   - the return value is an aria_q4_status; nothing aborts the process
 *     (the reference unwraps and aborts on any CUDA error, Cargo.toml:24);
 *   - layouts name the orientation of the reference's flat f16 tensor:
 *       ARIA_Q4_LAYOUT_KN  w[k][n], blocks run along n: w_qkv [d][3d],
 *                          w_out [d][d], w_ff1 [d][ff], w_ff2 [ff][d]
 *                          (src/transformer_cuda.rs:263-270, gemm(..,false,false))
 *       ARIA_Q4_LAYOUT_NK  w[n][k], blocks run along k: the tied LM head
 *                          embed [V][d] (src/transformer_cuda.rs:314, :1864,
 *                          gemm(..,false,true))
 */
#ifndef ARIA_Q4_H
#define ARIA_Q4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ARIA_Q4_ABI_VERSION 1

#if defined(__GNUC__)
#define ARIA_Q4_API __attribute__((visibility("default")))
#else
#define ARIA_Q4_API
#endif

typedef enum {
  ARIA_Q4_OK = 0,
  ARIA_Q4_EINVAL = 1,       /* null pointer, negative size, bad enum value        */
  ARIA_Q4_EUNSUPPORTED = 2, /* shape outside what the kernels handle (K % 32 etc.) */
  ARIA_Q4_EALIGN = 3,       /* pointer or leading dimension not 16-byte aligned   */
  ARIA_Q4_ECUDA = 4,        /* a CUDA runtime call failed: aria_q4_last_cuda_error */
  ARIA_Q4_ENODEVICE = 5,    /* current device is not an sm_100 (B200) GPU          */
  ARIA_Q4_ESIZE = 6         /* destination buffer smaller than required           */
} aria_q4_status;

enum { ARIA_Q4_LAYOUT_KN = 0, ARIA_Q4_LAYOUT_NK = 1 };
/* element types, numbered like the reference's GGUF dtype ids (:2853, :3213) */
enum { ARIA_Q4_F32 = 0, ARIA_Q4_F16 = 1 };

/* ---------------------------------------------------------------- packer */

/* Bytes of GGUF Q4_0 for n elements: ceil(n/32)*18 (src/transformer_cuda.rs:550-552). */
ARIA_Q4_API size_t aria_q4_0_packed_bytes(size_t n);

/* Replaces `quantize_q4_0(&[f32]) -> Vec<u8>` (src/transformer_cuda.rs:549-575) as
 * called by push_q4! (:3214-3218) on a downloaded f16 weight: src is n f16 values,
 * dst receives aria_q4_0_packed_bytes(n) bytes, identical to the Rust packer's. */
ARIA_Q4_API int aria_q4_0_pack_f16(const uint16_t* src, size_t n, uint8_t* dst, void* stream);

/* Same packer on an f32 buffer: the exact signature of quantize_q4_0 (&[f32]). */
ARIA_Q4_API int aria_q4_0_pack_f32(const float* src, size_t n, uint8_t* dst, void* stream);

/* Exact dequantisation (q-8)*scale of n elements of GGUF Q4_0 into f32.  The
 * reference has no dequantiser (it never reads Q4_0 back, :3046-3065); this is
 * the inverse its packer implies, used for checking and export round trips. */
ARIA_Q4_API int aria_q4_0_unpack_f32(const uint8_t* blocks, size_t n, float* dst, void* stream);

/* ---------------------------------------------------------------- device form */

/* Bytes of the device-resident ("tiled") form of a K x N projection. */
ARIA_Q4_API size_t aria_q4_0_tiled_bytes(int K, int N);

/* Uploads a Q4_0 GGUF tensor into the tiled form.  Stands where the reference
 * loader fills TransformerLayer.w_* / embed with f16 (load_f16!, :3046-3055),
 * which cannot read dtype 2.  `blocks` = the tensor's K*N/32*18 bytes in the
 * reference's flat order for `layout`.  Requires K % 32 == 0, and N % 32 == 0
 * for KN.  tiled must be 256-byte aligned (cudaMalloc memory is). */
ARIA_Q4_API int aria_q4_0_repack(const uint8_t* blocks, int layout, int K, int N,
                     void* tiled, size_t tiled_bytes, void* stream);

/* Quantises f16 weights (the reference's in-memory w_* / embed) straight into
 * the tiled form, with the same bit-exact block quantiser as aria_q4_0_pack_*:
 * repack(pack(w)) == quantize_tiled(w) byte for byte. */
ARIA_Q4_API int aria_q4_0_quantize_tiled(const uint16_t* w, int layout, int K, int N,
                             void* tiled, size_t tiled_bytes, void* stream);

/* ---------------------------------------------------------------- projection */

/* Replaces `gemm(blas, x, w, y, m, k, n, false, transb, alpha, beta)` followed
 * by `add_bias` (src/transformer_cuda.rs:615-640 with :1583/:1686/:1753/:1805/
 * :1864) when the weight is Q4_0:
 *     y[m][n] = alpha * sum_k x[m][k] * W(k,n) + beta * y[m][n] + bias[n]
 * W is the tiled form of the layout-oriented Q4_0 tensor (KN <=> transb=false,
 * NK <=> transb=true).  x is f16 [M][ldx]; y is f16 or f32 (y_dtype) [M][ldy];
 * bias (f16 [N]) may be NULL.  fp32 accumulation.  x must be 16-byte aligned
 * with ldx % 8 == 0.  M >= 0; M == 0 is a no-op. */
ARIA_Q4_API int aria_q4_0_matmul(const void* tiled, int layout, int K, int N,
                     const uint16_t* x, int M, int ldx,
                     void* y, int y_dtype, int ldy,
                     const uint16_t* bias, float alpha, float beta, void* stream);

/* Flags of aria_q4_0_matmul_ex. */
enum {
  /* The weight buffer is not written by the kernel that precedes this call on
   * the stream (true for model weights loaded at start-up).  The projection may
   * then read its weights before waiting for that kernel to finish, overlapping
   * weight streaming with the previous projection's tail.  Leave it clear when
   * the weights were just produced on the same stream (repack/quantize). */
  ARIA_Q4_FLAG_CONST_WEIGHTS = 1,
  /* Kernel selection (at most one; without any the library chooses).
   * STREAM: the streaming GEMV (M <= 8; each warp streams packed chunks through a
   * shared-memory ring; best for weights of tens of MB).  REGISTER: the
   * register-fed decode kernel (M <= 64; lowest latency for small weights).
   * ARIA_Q4_EUNSUPPORTED when the chosen kernel cannot take the shape. */
  ARIA_Q4_FLAG_KERNEL_STREAM = 2,
  ARIA_Q4_FLAG_KERNEL_REGISTER = 4,
  /* TENSOR: the tcgen05 tensor-core kernel (any M >= 1). */
  ARIA_Q4_FLAG_KERNEL_TENSOR = 8,
  /* Epilogue activation: y = gelu(alpha * x.W + bias) + beta * y, with the
   * reference's tanh-form GELU computed in f32 and one rounding to y's type.
   * Replaces the reference's add_bias + gelu_fwd launches after the ffn_up
   * projection (src/transformer_cuda.rs:1789-1794, src/kernels.cu:574-583),
   * which round to f16 after the GEMM, the bias add and the GELU. */
  ARIA_Q4_FLAG_EPILOGUE_GELU = 16
};

/* aria_q4_0_matmul with scheduling flags (ARIA_Q4_FLAG_*); flags = 0 is exactly
 * aria_q4_0_matmul.  No reference counterpart: a launch hint for chains of
 * projections (the reference's per-layer gemm() calls, :1583-:1864). */
ARIA_Q4_API int aria_q4_0_matmul_ex(const void* tiled, int layout, int K, int N,
                        const uint16_t* x, int M, int ldx,
                        void* y, int y_dtype, int ldy,
                        const uint16_t* bias, float alpha, float beta, int flags, void* stream);

/* Bytes of workspace with which aria_q4_0_matmul_ws may split K for this
 * shape (0: no split would help).  The workspace proposed for the reference's
 * gemm() replacement (`void* workspace, size_t ws_bytes`). */
ARIA_Q4_API size_t aria_q4_0_workspace_bytes(int K, int N, int M);

/* aria_q4_0_matmul_ex with a caller-owned device workspace (256-byte aligned;
 * NULL or 0 bytes: no K split).  When the tensor-core kernel has fewer output
 * tiles than SMs it splits K into work units whose f32 partials go to the
 * workspace; the last unit of each tile adds them in slice order (results are
 * reproducible).  The workspace must be zero-filled before its first use;
 * every call, of any shape, leaves it ready for the next -- except a call
 * during which a bounded wait expired (aria_q4_take_device_error() != 0):
 * zero the workspace's first aria_q4_0_workspace_counter_bytes() bytes
 * again before reusing it.  Calls that share a workspace must be ordered (one
 * stream, or events). */
ARIA_Q4_API int aria_q4_0_matmul_ws(const void* tiled, int layout, int K, int N,
                        const uint16_t* x, int M, int ldx,
                        void* y, int y_dtype, int ldy,
                        const uint16_t* bias, float alpha, float beta,
                        void* workspace, size_t workspace_bytes, int flags, void* stream);

/* Bytes at the start of every workspace that hold the split-K tile counters
 * (the region that must be zero before a call). */
ARIA_Q4_API size_t aria_q4_0_workspace_counter_bytes(void);

/* Kernels aria_q4_0_matmul_ws can run. */
enum {
  ARIA_Q4_KERNEL_STREAM = 1,    /* streaming GEMV (gemv_stream_kernel) */
  ARIA_Q4_KERNEL_REGISTER = 2,  /* register-fed decode kernel (decode_mma_kernel) */
  ARIA_Q4_KERNEL_TENSOR = 3     /* tcgen05 kernel (gemm_tc_kernel) */
};

/* The kernel aria_q4_0_matmul_ws would launch for this shape, a workspace of
 * workspace_bytes (0: none) and these flags; a negated status code when the
 * arguments would be rejected.  No reference counterpart (introspection for
 * benchmarks and tests). */
ARIA_Q4_API int aria_q4_0_kernel_choice(int layout, int K, int N, int M, size_t workspace_bytes, int flags);

/* aria_q4_0_matmul_ex for callers that cannot allocate device memory: those
 * that run inside another framework's memory pool or a captured CUDA graph
 * where cudaMalloc is not allowed, or that hold no allocator at all (a
 * foreign-language host calling through this C ABI).  Where the tensor-core
 * kernel splits K it uses the library's own static device scratch -- a
 * file-scope 8 MiB array that every GPU which loads the library holds until
 * the process exits -- in place of a caller workspace, choosing only splits
 * whose partials fit in it (a shape whose best split would need more runs with
 * a smaller split or none).  The call allocates nothing.  The first call on a
 * device looks up the array's device address once (cudaGetSymbolAddress), so
 * make it before any stream capture; that cached address does not survive
 * cudaDeviceReset.  Each call that splits K first clears the scratch's
 * counter region on the stream.  Every call on a device shares that one
 * scratch and it keeps the last call's contents: calls that overlap on the GPU
 * (unordered streams, or several host threads) race and corrupt each other's
 * partial sums, so order them on one stream.  No counterpart in the
 * reference. */
ARIA_Q4_API int aria_q4_0_matmul_static_ws(const void* tiled, int layout, int K, int N,
                        const uint16_t* x, int M, int ldx,
                        void* y, int y_dtype, int ldy,
                        const uint16_t* bias, float alpha, float beta, int flags, void* stream);

/* ---------------------------------------------------------------- decode step */

/* The rest of a decode step with KV cache, around the projections above.  The
 * reference runs its cached decode step on the CPU only (`step`,
 * src/transformer_cuda.rs:1286-1324, over cpu_layer_forward :1059-1166); these
 * kernels are its GPU counterparts.  The residual stream h is f32 [M][d] (the
 * projections add into it with y_dtype = ARIA_Q4_F32 and beta = 1); activations
 * fed to projections and the KV caches are f16. */

/* aria_q4_0_matmul_ex with the reference's LayerNorm as its prologue:
 *     y = act(alpha * LayerNorm(h) . W + bias) + beta * y
 * where LayerNorm(h) = (h - mean) / sqrt(var + eps) * gamma + beta_ln per f32
 * row of h [M][ldh] (two-pass statistics, rounded once to f16 -- the value a
 * separate LayerNorm would store for the projection to read).  Replaces the
 * reference's LayerNorm + gemm pairs before QKV and ffn_up (cpu_layer_forward
 * :1092-1096 and :1145-1150; LayerNorm :3271-3293, eps 1e-5) in one launch.
 * Runs the register-fed decode kernel: M <= 64; flags: CONST_WEIGHTS,
 * KERNEL_REGISTER, EPILOGUE_GELU.  h 16-byte aligned with ldh % 4 == 0;
 * gamma, beta_ln f16 [K], 16-byte aligned. */
ARIA_Q4_API int aria_q4_0_matmul_ln(const void* tiled, int layout, int K, int N, const float* h, int M, int ldh,
                                    const uint16_t* gamma, const uint16_t* beta_ln, float eps,
                                    void* y, int y_dtype, int ldy, const uint16_t* bias, float alpha, float beta,
                                    int flags, void* stream);

/* h[m] = embed[tokens[m]] + pos_embed[positions[m]] (f16 tables [vocab][d],
 * [max_seq][d]; f32 out), token and position clamped into the tables as the
 * reference clamps them (:1290-1297).  tokens, positions: device int [M]. */
ARIA_Q4_API int aria_embed_f16(const uint16_t* embed, const uint16_t* pos_embed, int vocab, int max_seq, int d,
                               const int* tokens, const int* positions, int M, float* h, void* stream);

/* y[m] = (x[m] - mean) / sqrt(var + eps) * gamma + beta over the d values of
 * each f32 row, f16 out with row stride ldy (cpu_layernorm, :3271-3293; the
 * reference uses eps = 1e-5).  d <= 8192. */
ARIA_Q4_API int aria_layernorm_f32(const float* x, int M, int d, const uint16_t* gamma, const uint16_t* beta,
                                   float eps, uint16_t* y, int ldy, void* stream);

/* Single-token attention of M sequences (the attention block of
 * cpu_layer_forward with t = 1, :1098-1137): qkv is f16 [M][3d] (q, k, v of the
 * new token, heads of d / heads dimensions); its k and v are written into the
 * caches (f16 [M][max_seq][d]) at positions[m] (device int [M]), then each
 * head attends over positions 0..positions[m] with scale 1/sqrt(d / heads)
 * and a max-subtracted softmax; out is f16 [M][d].  A position outside
 * [0, max_seq) writes nothing to the caches and zeros to its output row.
 * d / heads one of 32, 64, 128, 256; qkv and caches 16-byte aligned. */
ARIA_Q4_API int aria_attention_decode(const uint16_t* qkv, int M, int d, int heads, uint16_t* k_cache,
                                      uint16_t* v_cache, int max_seq, const int* positions, uint16_t* out,
                                      void* stream);

/* Causal attention over whole prompts on the tensor cores: the reference's
 * flash_attn_fwd (src/kernels.cu:1298-1437; q, k, v, out [NH][T][dh] f16,
 * lse [NH][T] f32) with the same arguments and meaning -- out[h][t] =
 * sum over s <= t of softmax_s(scale q[h][t].k[h][s]) v[h][s] and lse[h][t] =
 * max + ln(sum of exp) of that row (natural log).  lse may be NULL.  dh 64 or
 * 128; q, k, v, out 16-byte aligned.  NH = sequences x heads, T >= 1. */
ARIA_Q4_API int aria_flash_attn_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                                    float* lse, int NH, int T, int dh, float scale, void* stream);

/* The same attention read straight from the QKV projection's output: qkv is
 * f16 [B * T][3 d] (rows of sequence b at b T .. b T + T - 1; q, k, v of head
 * h at columns h dh, d + h dh, 2 d + h dh), out f16 [B * T][d] with the heads
 * side by side -- the layout attn_out reads (forward_gpu's attention block,
 * src/transformer_cuda.rs:1583-1686).  scale 1/sqrt(dh); lse [B][heads][T] or
 * NULL.  k_cache, v_cache (both or neither; f16 [B][max_seq][d], max_seq >= T):
 * the keys and values of positions 0 .. T - 1 are also stored there, as the
 * decode step's caches hold them (the reference's KVCache,
 * src/transformer_cuda.rs:144-155), in the same launch.  dh = d / heads 64 or
 * 128; d a multiple of 8; qkv, out and the caches 16-byte aligned. */
ARIA_Q4_API int aria_attention_prefill(const uint16_t* qkv, int B, int T, int d, int heads, uint16_t* out,
                                       float* lse, uint16_t* k_cache, uint16_t* v_cache, int max_seq, void* stream);

/* ---------------------------------------------------------------- multi-GPU */

/* The reduction of the column-split FFN over NVLink peer memory (BASELINE
 * configs[4] decode on 2..8 GPUs of one node): replaces an NCCL all-reduce of
 * the ranks' f32 ffn_down partials followed by the residual add.  No
 * reference counterpart (the reference runs on one device,
 * src/transformer_cuda.rs:83-103).
 *
 * Set-up (once, outside any stream capture): every rank allocates one region
 * with aria_p2p_alloc (zero-filled; the only allocating call of the library),
 * exports it with aria_p2p_ipc_handle, exchanges the 64-byte handles with its
 * peers (any host channel) and maps theirs with aria_p2p_ipc_open.  Each
 * region holds, at offsets the caller chooses, one f32 partial buffer per
 * layer, a flag block of 8 unsigned words and a state block of 2 words.
 *
 * aria_p2p_allreduce_add: h[0..n) (f16) += sum over ranks r of part[r][0..n)
 * (f32, rank order, identical bits on every rank), where part[r] is this
 * layer's partial buffer on rank r (the peers' through their mappings) and
 * flag[r] rank r's flag block; state is this rank's state block.  Every rank
 * must make the same sequence of calls (a call per layer, layers in order);
 * the partial of a layer must not be rewritten before the following call has
 * completed on this rank (one buffer per layer satisfies it).  The call
 * waits on the GPU (bounded by wait_limit_us, 1..10^7) for every peer's
 * partial of the same call; if one never arrives it records
 * ARIA_Q4_DEVERR_PEER_TIMEOUT, leaves h unchanged and returns.  nranks 1..8,
 * n a multiple of 8, h and the partials 16-byte aligned.  part and flag are
 * HOST arrays of nranks device pointers.  Stream-ordered; captured launches
 * stay correct on replay (the call counter lives in the state block). */
ARIA_Q4_API int aria_p2p_alloc(size_t bytes, void** ptr);
ARIA_Q4_API int aria_p2p_free(void* ptr);
ARIA_Q4_API int aria_p2p_ipc_handle(const void* ptr, void* handle /* 64 bytes */);
ARIA_Q4_API int aria_p2p_ipc_open(const void* handle /* 64 bytes */, void** ptr);
ARIA_Q4_API int aria_p2p_ipc_close(void* ptr);
ARIA_Q4_API int aria_p2p_allreduce_add(const float* const* part, unsigned* const* flag, unsigned* state, int nranks,
                                       int rank, uint16_t* h, int n, unsigned wait_limit_us, void* stream);

/* ---------------------------------------------------------------- errors */

ARIA_Q4_API const char* aria_q4_strerror(int status);
/* cudaError_t of the last failing CUDA call on this thread (0 if none). */
ARIA_Q4_API int aria_q4_last_cuda_error(void);
/* Device-side error codes (aria_q4_take_device_error). */
enum {
  ARIA_Q4_DEVERR_NONE = 0,
  ARIA_Q4_DEVERR_TIMEOUT_FULL = 1,   /* the MMA issuer waited too long for an operand stage */
  ARIA_Q4_DEVERR_TIMEOUT_EMPTY = 2,  /* a producer waited too long for a free stage */
  ARIA_Q4_DEVERR_TIMEOUT_ACCUM = 3,  /* an accumulator hand-off waited too long */
  ARIA_Q4_DEVERR_PEER_TIMEOUT = 4    /* aria_p2p_allreduce_add: a peer never published its partial */
};

/* Reads and clears the device-side error code of the current device: 0 = none,
 * ARIA_Q4_DEVERR_* = a bounded wait inside a kernel expired (the tcgen05
 * kernels record the first such wait, unwind and return without finishing
 * their tiles instead of hanging; the peer reduction leaves h unchanged),
 * -1 = the read failed.  One code per device,
 * shared by every stream and thread.  Synchronises the device.  No reference
 * counterpart (the reference aborts). */
ARIA_Q4_API int aria_q4_take_device_error(void);
ARIA_Q4_API int aria_q4_abi_version(void);

/* ---------------------------------------------------------------- test hook */

/* Runs the tcgen05 kernel (no K split) with its activation-tile producer
 * issuing no copies and every pipeline wait limited to wait_limit_us
 * (1..1000000): the MMA issuer's first wait then runs out, the kernel records
 * ARIA_Q4_DEVERR_TIMEOUT_FULL, releases its tensor memory and returns, and y
 * is left unspecified.  Exists so that tests can drive the failure path
 * without faulting the GPU; no reference counterpart. */
ARIA_Q4_API int aria_q4_test_tensor_stall(const void* tiled, int layout, int K, int N,
                        const uint16_t* x, int M, int ldx,
                        void* y, int y_dtype, int ldy, unsigned wait_limit_us, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ARIA_Q4_H */
