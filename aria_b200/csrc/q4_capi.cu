// q4_capi.cu -- extern "C" entry points of libaria_q4.so (declared in
// include/aria_q4.h).  Argument checking, status codes and kernel selection;
// the kernels live in q4_pack.cu, q4_gemv.cu, q4_decode.cu and q4_gemm_tc.cu.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/aria_q4.h"
#include "q4_common.cuh"

namespace aria_q4 {
cudaError_t launch_pack_f16(const uint16_t* src, size_t n, uint8_t* dst, cudaStream_t st);
cudaError_t launch_pack_f32(const float* src, size_t n, uint8_t* dst, cudaStream_t st);
cudaError_t launch_unpack(const uint8_t* blocks, size_t n, float* dst, cudaStream_t st);
cudaError_t launch_repack(const uint8_t* blocks, int layout, int K, int N, uint8_t* tiled, cudaStream_t st);
cudaError_t launch_quantize_tiled(const uint16_t* w, int layout, int K, int N, uint8_t* tiled, cudaStream_t st);
cudaError_t launch_decode(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                          int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl,
                          bool const_weights, const float* ln_h = nullptr, const __half* ln_g = nullptr,
                          const __half* ln_b = nullptr, float ln_eps = 0.0f);
bool gemv_supported(int K, int N, int M);
cudaError_t launch_gemv(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                        int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl,
                        bool const_weights);
cudaError_t launch_gemm_tc(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                           int ydt, int ldy, const __half* bias, float alpha, float beta, void* workspace,
                           size_t workspace_bytes, cudaStream_t st, bool pdl, bool const_weights,
                           unsigned long long wait_ns = 1000000000ull, bool no_x_loads = false);
size_t tc_workspace_bytes(int K, int N, int M);
size_t tc_workspace_used(int K, int N, int M, size_t ws_avail);
size_t tc_workspace_counter_bytes();
int take_device_error();
int attn_take_device_error();
int p2p_take_device_error();
cudaError_t launch_p2p_allreduce(const float* const* part, unsigned* const* flag, unsigned* state, int nranks,
                                 int rank, __half* h, int n, unsigned long long wait_ns, cudaStream_t st);
cudaError_t launch_attention_prefill(const __half* q, const __half* k, const __half* v, int DH, long long s_head,
                                     long long s_pos, long long s_seq, int B, int H, int T, float scale, __half* out,
                                     long long o_seq, long long o_head, long long o_pos, float* lse,
                                     __half* k_cache, __half* v_cache, int max_seq, cudaStream_t st);
cudaError_t launch_embed(const __half* embed, const __half* pos_embed, const int* tok, const int* pos, int M, int vocab,
                         int max_seq, int d, float* h, cudaStream_t st);
cudaError_t launch_layernorm(const float* x, const __half* g, const __half* b, int M, int d, float eps, __half* y,
                             int ldy, cudaStream_t st);
size_t attention_smem_bytes(int dh, int max_seq);
cudaError_t launch_attention(const __half* qkv, int M, int d, int heads, int max_seq, const int* pos, __half* kc,
                             __half* vc, __half* out, cudaStream_t st);
}  // namespace aria_q4

// M at or below which the register-fed decode kernel is used; above it the
// tcgen05 kernel (each dequantised weight then serves up to 256 tokens).
#ifndef ARIA_Q4_DECODE_MAX_M
#define ARIA_Q4_DECODE_MAX_M 64
#endif
static const int kDecodeMaxM = ARIA_Q4_DECODE_MAX_M;

// Default decode-kernel choice: the streaming GEMV for M <= 8 when the weight
// is at least kStreamMinBytesPerSm of packed bytes per SM, or K is tall (the
// register-fed kernel then needs clusters to split K; measured on the Efkolos
// ffn_down, K = 3584: 4.0 against 4.4 us per chained launch).  Below that a
// projection is latency-bound and the register-fed kernel, with its smaller
// CTAs, overlaps better with its neighbours in a chain of projections.
static const double kStreamMinBytesPerSm = 32.0 * 1024;
static const int kStreamMinK = 2048;
static const int kRegisterMaxN = 1024;
static bool stream_by_default(int K, int N, int M) {
  if (M > 8) return false;
  const double per_sm = (double)N * (aria_q4::padded_k(K) / 128) * 72.0 / 148.0;
  return (per_sm >= kStreamMinBytesPerSm || K >= kStreamMinK) && aria_q4::gemv_supported(K, N, M);
}

using namespace aria_q4;

static thread_local int g_last_cuda_error = 0;

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return ARIA_Q4_OK;
  g_last_cuda_error = (int)e;
  return ARIA_Q4_ECUDA;
}

// The library is built for sm_100a only; refuse to launch anywhere else.
static int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  int major = 0, minor = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return cuda_status(e);
  e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (major != 10 || minor != 0) return ARIA_Q4_ENODEVICE;
  return ARIA_Q4_OK;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static int check_tiled_shape(int layout, int K, int N) {
  if (layout != ARIA_Q4_LAYOUT_KN && layout != ARIA_Q4_LAYOUT_NK) return ARIA_Q4_EINVAL;
  if (K <= 0 || N <= 0) return ARIA_Q4_EINVAL;
  if (K % kBlock != 0) return ARIA_Q4_EUNSUPPORTED;
  if (layout == ARIA_Q4_LAYOUT_KN && N % kBlock != 0) return ARIA_Q4_EUNSUPPORTED;
  if ((long long)K * (long long)N >= (1LL << 40)) return ARIA_Q4_EUNSUPPORTED;
  return ARIA_Q4_OK;
}

extern "C" {

size_t aria_q4_0_packed_bytes(size_t n) { return (n + kBlock - 1) / kBlock * kBlockBytes; }

int aria_q4_0_pack_f16(const uint16_t* src, size_t n, uint8_t* dst, void* stream) {
  if (n == 0) return ARIA_Q4_OK;
  if (!src || !dst) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_pack_f16(src, n, dst, (cudaStream_t)stream));
}

int aria_q4_0_pack_f32(const float* src, size_t n, uint8_t* dst, void* stream) {
  if (n == 0) return ARIA_Q4_OK;
  if (!src || !dst) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_pack_f32(src, n, dst, (cudaStream_t)stream));
}

int aria_q4_0_unpack_f32(const uint8_t* blocks, size_t n, float* dst, void* stream) {
  if (n == 0) return ARIA_Q4_OK;
  if (!blocks || !dst) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_unpack(blocks, n, dst, (cudaStream_t)stream));
}

size_t aria_q4_0_tiled_bytes(int K, int N) {
  if (K <= 0 || N <= 0) return 0;
  return tiled_bytes(K, N);
}

int aria_q4_0_repack(const uint8_t* blocks, int layout, int K, int N, void* tiled, size_t tiled_bytes_,
                     void* stream) {
  if (int s = check_tiled_shape(layout, K, N)) return s;
  if (!blocks || !tiled) return ARIA_Q4_EINVAL;
  if (((uintptr_t)tiled & 255u) != 0) return ARIA_Q4_EALIGN;
  if (tiled_bytes_ < tiled_bytes(K, N)) return ARIA_Q4_ESIZE;
  if (int s = check_device()) return s;
  return cuda_status(launch_repack(blocks, layout, K, N, (uint8_t*)tiled, (cudaStream_t)stream));
}

int aria_q4_0_quantize_tiled(const uint16_t* w, int layout, int K, int N, void* tiled, size_t tiled_bytes_,
                             void* stream) {
  if (int s = check_tiled_shape(layout, K, N)) return s;
  if (!w || !tiled) return ARIA_Q4_EINVAL;
  if (((uintptr_t)tiled & 255u) != 0) return ARIA_Q4_EALIGN;
  if (tiled_bytes_ < tiled_bytes(K, N)) return ARIA_Q4_ESIZE;
  if (int s = check_device()) return s;
  return cuda_status(launch_quantize_tiled(w, layout, K, N, (uint8_t*)tiled, (cudaStream_t)stream));
}

// Kernel choice: the streaming GEMV for M <= 8 and large weights; the
// register-fed decode kernel up to 32 tokens, and up to 64 when the weight has
// at most kRegisterMaxN outputs (few row tiles: its 16-token passes beat the
// tcgen05 kernel's fixed cost; measured on B200 in chains at M = 64: Efkolos
// attn_out 2.8 against 6.5 us, ffn_down 10.3 against 12.4 us); the tcgen05
// kernel above that (splitting K through the workspace when tiles are few),
// except without a workspace for the shapes it would have split (the
// register-fed kernel splits K itself).  ARIA_Q4_FLAG_KERNEL_* overrides the
// choice.  Returns an ARIA_Q4_KERNEL_* value, or a negated status.
static int choose_kernel(int K, int N, int M, bool has_workspace, int flags) {
  const bool want_stream = (flags & ARIA_Q4_FLAG_KERNEL_STREAM) != 0;
  const bool want_register = (flags & ARIA_Q4_FLAG_KERNEL_REGISTER) != 0;
  const bool want_tensor = (flags & ARIA_Q4_FLAG_KERNEL_TENSOR) != 0;
  if ((int)want_stream + (int)want_register + (int)want_tensor > 1) return -ARIA_Q4_EINVAL;
  if (want_stream) return gemv_supported(K, N, M) ? ARIA_Q4_KERNEL_STREAM : -ARIA_Q4_EUNSUPPORTED;
  if (want_register) return M <= kDecodeMaxM ? ARIA_Q4_KERNEL_REGISTER : -ARIA_Q4_EUNSUPPORTED;
  if (want_tensor) return ARIA_Q4_KERNEL_TENSOR;
  if (stream_by_default(K, N, M)) return ARIA_Q4_KERNEL_STREAM;
  if (M <= 32 || (M <= kDecodeMaxM && (N <= kRegisterMaxN || (!has_workspace && tc_workspace_bytes(K, N, M) > 0))))
    return ARIA_Q4_KERNEL_REGISTER;
  return ARIA_Q4_KERNEL_TENSOR;
}

size_t aria_q4_0_workspace_bytes(int K, int N, int M) {
  if (check_tiled_shape(ARIA_Q4_LAYOUT_NK, K, N) != ARIA_Q4_OK || M <= 32) return 0;
  return tc_workspace_bytes(K, N, M);
}

// Arguments shared by every projection entry point; ARIA_Q4_OK when a launch
// may follow (M == 0 also returns ARIA_Q4_OK: the caller then launches nothing).
static int check_matmul_args(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx,
                             const void* y, int y_dtype, int ldy, int flags) {
  if (int s = check_tiled_shape(layout, K, N)) return s;
  if (M < 0) return ARIA_Q4_EINVAL;
  if (M == 0) return ARIA_Q4_OK;
  if (!tiled || !x || !y) return ARIA_Q4_EINVAL;
  if (y_dtype != ARIA_Q4_F16 && y_dtype != ARIA_Q4_F32) return ARIA_Q4_EINVAL;
  if (ldx < K || ldy < N) return ARIA_Q4_EINVAL;
  const int known = ARIA_Q4_FLAG_CONST_WEIGHTS | ARIA_Q4_FLAG_KERNEL_STREAM | ARIA_Q4_FLAG_KERNEL_REGISTER |
                    ARIA_Q4_FLAG_KERNEL_TENSOR | ARIA_Q4_FLAG_EPILOGUE_GELU;
  if ((flags & ~known) != 0) return ARIA_Q4_EINVAL;
  if (((uintptr_t)tiled & 255u) != 0 || !aligned16(x) || (ldx % 8) != 0) return ARIA_Q4_EALIGN;
  return ARIA_Q4_OK;
}

int aria_q4_0_matmul_ws(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx, void* y,
                        int y_dtype, int ldy, const uint16_t* bias, float alpha, float beta, void* workspace,
                        size_t workspace_bytes, int flags, void* stream) {
  if (int s = check_matmul_args(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, flags)) return s;
  if (M == 0) return ARIA_Q4_OK;
  if (workspace_bytes == 0) workspace = nullptr;
  if (workspace && ((uintptr_t)workspace & 255u) != 0) return ARIA_Q4_EALIGN;
  if (int s = check_device()) return s;
  const cudaStream_t st = (cudaStream_t)stream;
  const int kern = choose_kernel(K, N, M, workspace != nullptr, flags);
  if (kern < 0) return -kern;
  const bool cw = (flags & ARIA_Q4_FLAG_CONST_WEIGHTS) != 0;
  // the kernels' output code: dtype in bit 0, GELU epilogue in bit 1 (aria_q4::kOutGelu)
  const int out = y_dtype | ((flags & ARIA_Q4_FLAG_EPILOGUE_GELU) ? aria_q4::kOutGelu : 0);
  if (kern == ARIA_Q4_KERNEL_STREAM)
    return cuda_status(launch_gemv((const uint8_t*)tiled, layout, K, N, (const __half*)x, M, ldx, y, out, ldy,
                                   (const __half*)bias, alpha, beta, st, true, cw));
  if (kern == ARIA_Q4_KERNEL_REGISTER)
    return cuda_status(launch_decode((const uint8_t*)tiled, layout, K, N, (const __half*)x, M, ldx, y, out, ldy,
                                     (const __half*)bias, alpha, beta, st, true, cw));
  return cuda_status(launch_gemm_tc((const uint8_t*)tiled, layout, K, N, (const __half*)x, M, ldx, y, out, ldy,
                                    (const __half*)bias, alpha, beta, workspace, workspace_bytes, st, true, cw));
}

size_t aria_q4_0_workspace_counter_bytes(void) { return tc_workspace_counter_bytes(); }

int aria_q4_0_kernel_choice(int layout, int K, int N, int M, size_t workspace_bytes, int flags) {
  if (int s = check_tiled_shape(layout, K, N)) return -s;
  if (M < 1) return -ARIA_Q4_EINVAL;
  const int known = ARIA_Q4_FLAG_CONST_WEIGHTS | ARIA_Q4_FLAG_KERNEL_STREAM | ARIA_Q4_FLAG_KERNEL_REGISTER |
                    ARIA_Q4_FLAG_KERNEL_TENSOR | ARIA_Q4_FLAG_EPILOGUE_GELU;
  if ((flags & ~known) != 0) return -ARIA_Q4_EINVAL;
  return choose_kernel(K, N, M, workspace_bytes != 0, flags);
}

int aria_q4_0_matmul_ex(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx, void* y,
                        int y_dtype, int ldy, const uint16_t* bias, float alpha, float beta, int flags, void* stream) {
  return aria_q4_0_matmul_ws(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, bias, alpha, beta, nullptr, 0, flags,
                             stream);
}

// ------------------------------------------------------------------ static-scratch variant
// Scratch of aria_q4_0_matmul_static_ws: one file-scope device array per
// device (zero at module load), so the call allocates nothing.  Its first
// bytes are the split-K counter region, the rest the f32 partials.
static constexpr size_t kStaticWsBytes = 8u << 20;
static __device__ __align__(256) unsigned char g_static_ws[kStaticWsBytes];

// Device address of g_static_ws on the current device, looked up once per
// device (the first call on a device, which should therefore come before any
// stream capture); nullptr (and *err set) when the lookup fails.  The cache
// assumes the device's context lives as long as the process: after
// cudaDeviceReset the module, and with it the array, may be reloaded elsewhere.
static void* static_ws_address(cudaError_t* err) {
  constexpr int kMaxDevices = 64;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && (dev < 0 || dev >= kMaxDevices)) e = cudaErrorInvalidDevice;
  if (e != cudaSuccess) {
    *err = e;
    return nullptr;
  }
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_ws);
    if (e != cudaSuccess) {
      *err = e;
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

int aria_q4_0_matmul_static_ws(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx,
                               void* y, int y_dtype, int ldy, const uint16_t* bias, float alpha, float beta,
                               int flags, void* stream) {
  if (int s = check_matmul_args(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, flags)) return s;
  if (M == 0) return ARIA_Q4_OK;
  // The kernel and K split the library picks with kStaticWsBytes of workspace:
  // the tensor-core planner only considers splits whose partials fit, so every
  // shape runs (with a smaller split, or none, where the best one would not fit).
  const int kern = choose_kernel(K, N, M, true, flags);
  if (kern < 0) return -kern;
  const bool splits = kern == ARIA_Q4_KERNEL_TENSOR && tc_workspace_used(K, N, M, kStaticWsBytes) > 0;
  if (!splits)
    return aria_q4_0_matmul_ws(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, bias, alpha, beta, nullptr, 0,
                               flags, stream);
  cudaError_t e = cudaSuccess;
  void* ws = static_ws_address(&e);
  if (!ws) return cuda_status(e);
  // the split-K counters must start at zero (a call cut short by an expired
  // bounded wait may leave some set)
  e = cudaMemsetAsync(ws, 0, tc_workspace_counter_bytes(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e);
  return aria_q4_0_matmul_ws(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, bias, alpha, beta, ws, kStaticWsBytes,
                             flags, stream);
}

// ------------------------------------------------------------------ LayerNorm prologue
int aria_q4_0_matmul_ln(const void* tiled, int layout, int K, int N, const float* h, int M, int ldh,
                        const uint16_t* gamma, const uint16_t* beta_ln, float eps, void* y, int y_dtype, int ldy,
                        const uint16_t* bias, float alpha, float beta, int flags, void* stream) {
  if (int s = check_tiled_shape(layout, K, N)) return s;
  if (M < 0 || !(eps >= 0.0f)) return ARIA_Q4_EINVAL;
  if (M == 0) return ARIA_Q4_OK;
  if (!tiled || !h || !gamma || !beta_ln || !y) return ARIA_Q4_EINVAL;
  if (y_dtype != ARIA_Q4_F16 && y_dtype != ARIA_Q4_F32) return ARIA_Q4_EINVAL;
  if (ldh < K || ldy < N) return ARIA_Q4_EINVAL;
  const int known = ARIA_Q4_FLAG_CONST_WEIGHTS | ARIA_Q4_FLAG_KERNEL_REGISTER | ARIA_Q4_FLAG_EPILOGUE_GELU;
  if ((flags & ~known) != 0) return ARIA_Q4_EINVAL;
  if (M > kDecodeMaxM) return ARIA_Q4_EUNSUPPORTED;
  if (((uintptr_t)tiled & 255u) != 0 || !aligned16(h) || (ldh % 4) != 0 || !aligned16(gamma) || !aligned16(beta_ln))
    return ARIA_Q4_EALIGN;
  if (int s = check_device()) return s;
  const int out = y_dtype | ((flags & ARIA_Q4_FLAG_EPILOGUE_GELU) ? aria_q4::kOutGelu : 0);
  return cuda_status(launch_decode((const uint8_t*)tiled, layout, K, N, nullptr, M, ldh, y, out, ldy,
                                   (const __half*)bias, alpha, beta, (cudaStream_t)stream, true,
                                   (flags & ARIA_Q4_FLAG_CONST_WEIGHTS) != 0, h, (const __half*)gamma,
                                   (const __half*)beta_ln, eps));
}

// ------------------------------------------------------------------ decode-step helpers
int aria_embed_f16(const uint16_t* embed, const uint16_t* pos_embed, int vocab, int max_seq, int d,
                   const int* tokens, const int* positions, int M, float* h, void* stream) {
  if (M < 0 || d <= 0 || vocab <= 0 || max_seq <= 0) return ARIA_Q4_EINVAL;
  if (M == 0) return ARIA_Q4_OK;
  if (!embed || !pos_embed || !tokens || !positions || !h) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_embed((const __half*)embed, (const __half*)pos_embed, tokens, positions, M, vocab, max_seq,
                                  d, h, (cudaStream_t)stream));
}

int aria_layernorm_f32(const float* x, int M, int d, const uint16_t* gamma, const uint16_t* beta, float eps,
                       uint16_t* y, int ldy, void* stream) {
  if (M < 0 || d <= 0 || d > 32 * 256 || ldy < d || !(eps >= 0.0f)) return ARIA_Q4_EINVAL;
  if (M == 0) return ARIA_Q4_OK;
  if (!x || !gamma || !beta || !y) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_layernorm(x, (const __half*)gamma, (const __half*)beta, M, d, eps, (__half*)y, ldy,
                                      (cudaStream_t)stream));
}

int aria_attention_decode(const uint16_t* qkv, int M, int d, int heads, uint16_t* k_cache, uint16_t* v_cache,
                          int max_seq, const int* positions, uint16_t* out, void* stream) {
  if (M < 0 || d <= 0 || heads <= 0 || d % heads != 0 || max_seq <= 0) return ARIA_Q4_EINVAL;
  const int dh = d / heads;
  if (dh != 32 && dh != 64 && dh != 128 && dh != 256) return ARIA_Q4_EUNSUPPORTED;
  if (attention_smem_bytes(dh, max_seq) > 227 * 1024) return ARIA_Q4_EUNSUPPORTED;
  if (M == 0) return ARIA_Q4_OK;
  if (!qkv || !k_cache || !v_cache || !positions || !out) return ARIA_Q4_EINVAL;
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache)) return ARIA_Q4_EALIGN;
  if (int s = check_device()) return s;
  return cuda_status(launch_attention((const __half*)qkv, M, d, heads, max_seq, positions, (__half*)k_cache,
                                      (__half*)v_cache, (__half*)out, (cudaStream_t)stream));
}

int aria_flash_attn_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, float* lse, int NH,
                        int T, int dh, float scale, void* stream) {
  if (NH < 0 || T < 0 || !(scale == scale)) return ARIA_Q4_EINVAL;
  if (dh != 64 && dh != 128) return ARIA_Q4_EUNSUPPORTED;
  if (NH == 0 || T == 0) return ARIA_Q4_OK;
  if (!q || !k || !v || !out) return ARIA_Q4_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return ARIA_Q4_EALIGN;
  if ((long long)NH * ((T + 127) / 128) > 0x7fffffffLL) return ARIA_Q4_ESIZE;
  if (int s = check_device()) return s;
  // [NH][T][dh]: one head per "sequence" of the kernel's 4-D view
  const long long st = (long long)T * dh;
  return cuda_status(launch_attention_prefill((const __half*)q, (const __half*)k, (const __half*)v, dh, dh, dh, st,
                                              NH, 1, T, scale, (__half*)out, st, 0, dh, lse, nullptr, nullptr, 0,
                                              (cudaStream_t)stream));
}

int aria_attention_prefill(const uint16_t* qkv, int B, int T, int d, int heads, uint16_t* out, float* lse,
                           uint16_t* k_cache, uint16_t* v_cache, int max_seq, void* stream) {
  if (B < 0 || T < 0 || d <= 0 || heads <= 0 || d % heads != 0 || d % 8 != 0) return ARIA_Q4_EINVAL;
  const int dh = d / heads;
  if (dh != 64 && dh != 128) return ARIA_Q4_EUNSUPPORTED;
  if ((k_cache == nullptr) != (v_cache == nullptr)) return ARIA_Q4_EINVAL;
  if (k_cache && max_seq < T) return ARIA_Q4_ESIZE;
  if (B == 0 || T == 0) return ARIA_Q4_OK;
  if (!qkv || !out) return ARIA_Q4_EINVAL;
  if (!aligned16(qkv) || !aligned16(out)) return ARIA_Q4_EALIGN;
  if (k_cache && (!aligned16(k_cache) || !aligned16(v_cache))) return ARIA_Q4_EALIGN;
  if ((long long)B * heads * ((T + 127) / 128) > 0x7fffffffLL) return ARIA_Q4_ESIZE;
  if (int s = check_device()) return s;
  const __half* q = (const __half*)qkv;
  const long long row = 3LL * d;
  return cuda_status(launch_attention_prefill(q, q + d, q + 2 * d, dh, dh, row, row * T, B, heads, T,
                                              1.0f / sqrtf((float)dh), (__half*)out, (long long)T * d, dh, d, lse,
                                              (__half*)k_cache, (__half*)v_cache, max_seq, (cudaStream_t)stream));
}

// ------------------------------------------------------------------ failure-path test hook
int aria_q4_test_tensor_stall(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx,
                              void* y, int y_dtype, int ldy, unsigned wait_limit_us, void* stream) {
  if (int s = check_matmul_args(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, 0)) return s;
  if (M == 0) return ARIA_Q4_OK;
  if (wait_limit_us == 0 || wait_limit_us > 1000000u) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  return cuda_status(launch_gemm_tc((const uint8_t*)tiled, layout, K, N, (const __half*)x, M, ldx, y, y_dtype, ldy,
                                    nullptr, 1.0f, 0.0f, nullptr, 0, (cudaStream_t)stream, false, false,
                                    (unsigned long long)wait_limit_us * 1000ull, true));
}

int aria_q4_0_matmul(const void* tiled, int layout, int K, int N, const uint16_t* x, int M, int ldx, void* y,
                     int y_dtype, int ldy, const uint16_t* bias, float alpha, float beta, void* stream) {
  return aria_q4_0_matmul_ex(tiled, layout, K, N, x, M, ldx, y, y_dtype, ldy, bias, alpha, beta, 0, stream);
}

const char* aria_q4_strerror(int status) {
  switch (status) {
    case ARIA_Q4_OK: return "ok";
    case ARIA_Q4_EINVAL: return "invalid argument";
    case ARIA_Q4_EUNSUPPORTED: return "unsupported shape (K must be a multiple of 32; N too for layout KN)";
    case ARIA_Q4_EALIGN: return "misaligned pointer or leading dimension (x 16 B, ldx % 8, tiled 256 B)";
    case ARIA_Q4_ECUDA: return "CUDA runtime error (see aria_q4_last_cuda_error)";
    case ARIA_Q4_ENODEVICE: return "current device is not sm_100 (B200)";
    case ARIA_Q4_ESIZE: return "destination buffer too small";
    default: return "unknown status";
  }
}

int aria_q4_last_cuda_error(void) { return g_last_cuda_error; }

int aria_q4_take_device_error(void) {
  const int a = take_device_error();
  const int b = attn_take_device_error();
  const int c = p2p_take_device_error();
  return a != 0 ? a : b != 0 ? b : c;
}

// ------------------------------------------------------------------ peer reduction
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");

int aria_p2p_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return ARIA_Q4_EINVAL;
  if (int s = check_device()) return s;
  void* p = nullptr;
  if (cudaError_t e = cudaMalloc(&p, bytes)) return cuda_status(e);
  if (cudaError_t e = cudaMemset(p, 0, bytes)) {
    cudaFree(p);
    return cuda_status(e);
  }
  *ptr = p;
  return ARIA_Q4_OK;
}

int aria_p2p_free(void* ptr) { return ptr ? cuda_status(cudaFree(ptr)) : ARIA_Q4_OK; }

int aria_p2p_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return ARIA_Q4_EINVAL;
  cudaIpcMemHandle_t h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr))) return cuda_status(e);
  memcpy(handle, &h, sizeof(h));
  return ARIA_Q4_OK;
}

int aria_p2p_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return ARIA_Q4_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int aria_p2p_ipc_close(void* ptr) { return ptr ? cuda_status(cudaIpcCloseMemHandle(ptr)) : ARIA_Q4_EINVAL; }

int aria_p2p_allreduce_add(const float* const* part, unsigned* const* flag, unsigned* state, int nranks, int rank,
                           uint16_t* h, int n, unsigned wait_limit_us, void* stream) {
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks || n < 0 || n % 8 != 0) return ARIA_Q4_EINVAL;
  if (wait_limit_us == 0 || wait_limit_us > 10000000u) return ARIA_Q4_EINVAL;
  if (!part || !flag || !state || !h) return ARIA_Q4_EINVAL;
  for (int r = 0; r < nranks; r++) {
    if (!part[r] || !flag[r]) return ARIA_Q4_EINVAL;
    if (!aligned16(part[r]) || ((uintptr_t)flag[r] & 3u) != 0) return ARIA_Q4_EALIGN;
  }
  if (!aligned16(h) || ((uintptr_t)state & 7u) != 0) return ARIA_Q4_EALIGN;
  if (n == 0) return ARIA_Q4_OK;
  if (int s = check_device()) return s;
  return cuda_status(launch_p2p_allreduce(part, flag, state, nranks, rank, (__half*)h, n,
                                          (unsigned long long)wait_limit_us * 1000ull, (cudaStream_t)stream));
}
int aria_q4_abi_version(void) { return ARIA_Q4_ABI_VERSION; }

}  // extern "C"
