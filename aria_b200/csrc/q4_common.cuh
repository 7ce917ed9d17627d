// q4_common.cuh -- shared definitions for the B200 Q4_0 projection library.
//
// Two byte formats exist:
//
//  * GGUF Q4_0 blocks ("AoS"), exactly as ARIA's quantize_q4_0 writes them
//    (lold3344/ARIA src/transformer_cuda.rs:548-575): 18 bytes per 32 weights,
//    f16 scale little-endian first, then 16 bytes of nibbles, element 2j in the
//    low nibble of byte j and element 2j+1 in the high nibble.  Blocks run along
//    the flat storage order of the reference tensor, which is w[k][n] (KN) for
//    w_qkv/w_out/w_ff1/w_ff2 and embed[n][k] (NK) for the tied LM head.
//
//  * The device-resident "tiled" form the kernels read.  The 18-byte blocks are
//    not 16-byte aligned, so the loader splits them into two planes over a K
//    padded to Kp = roundup(K, 128) (padding codes are 8, padding scales 0):
//      qs     u8  [N][Kp/2]  output-feature-major: row n holds the 4-bit codes of
//                            W(:, n).  Each 128-k group of a row is 64 bytes =
//                            16 words; word 4t+i (t, i in 0..3) holds the 8
//                            consecutive k = 128G + 32i + 8t + (0..7).  A lane
//                            that owns "t" therefore reads its 8-k slice of all
//                            four 32-k blocks with one 16-byte load, and the
//                            four lanes t = 0..3 of a row read 64 contiguous bytes.
//      scales f16 NK: [Kp/128][N][4]  (one per (n, 32-k block), group-major: the four
//                                  block scales of a row's 128-k group are 8 contiguous
//                                  bytes and consecutive rows are adjacent)
//                 KN: [N/32][Kp]   (one per (k, 32-n block), transposed so that a
//                                   32-row group reads its k scales contiguously)
//    qs starts at byte 0, scales at align256(N*Kp/2).  Inside every 32-bit word
//    (8 consecutive k: e0..e7) the nibbles are stored in the order
//    e0 e2 e4 e6 e1 e3 e5 e7 (nibble 0 = bits 0..3), so that one LOP3 against
//    0x000F000F yields the f16x2 pair (e0, e1) with the 0x6400 exponent trick.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace aria_q4 {

constexpr int kBlock = 32;
constexpr int kBlockBytes = 18;

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline int padded_k(int K) { return (K + 127) / 128 * 128; }
__host__ __device__ inline size_t qs_row_bytes(int K) { return (size_t)padded_k(K) / 2; }

// byte offset of the scale plane inside a tiled buffer
__host__ __device__ inline size_t tiled_scale_offset(int K, int N) {
  return align_up((size_t)N * qs_row_bytes(K), 256);
}
__host__ __device__ inline size_t tiled_bytes(int K, int N) {
  return tiled_scale_offset(K, N) + (size_t)N * (size_t)padded_k(K) / 16;
}

// word (32-bit) index inside a qs row of the 8-k run starting at k (k % 8 == 0)
__host__ __device__ inline int qs_word_of_k(int k) {
  return 16 * (k >> 7) + 4 * ((k & 31) >> 3) + ((k & 127) >> 5);
}
// first k of word w of a row
__host__ __device__ inline int qs_k_of_word(int w) { return 128 * (w >> 4) + 32 * (w & 3) + 8 * ((w >> 2) & 3); }

// position of element i (0..7 of a word) inside the device word
__host__ __device__ inline int dev_nibble_pos(int i) { return (i >> 1) + 4 * (i & 1); }

// Pack 8 codes (element order) into one device word.
__host__ __device__ inline uint32_t dev_word_from_codes(const uint8_t* q8) {
  uint32_t w = 0;
#ifdef __CUDA_ARCH__
#pragma unroll
#endif
  for (int i = 0; i < 8; i++) w |= (uint32_t)(q8[i] & 0xF) << (4 * dev_nibble_pos(i));
  return w;
}

// Convert one reference-order word (byte j: low = e2j, high = e2j+1) into the
// device order.  Pure bit shuffling, used by the repack kernels.
__device__ __forceinline__ uint32_t ref_word_to_dev(uint32_t r) {
  // reference nibble p holds element p; device nibble dev_nibble_pos(i) holds element i.
  uint32_t even = r & 0x0F0F0F0Fu;         // e0 e2 e4 e6 at nibbles 0,2,4,6
  uint32_t odd = (r >> 4) & 0x0F0F0F0Fu;   // e1 e3 e5 e7 at nibbles 0,2,4,6
  // compact nibbles 0,2,4,6 -> 0,1,2,3 with byte permutes: pairs of bytes first
  even = (even | (even >> 4)) & 0x00FF00FFu;  // e0e2 in byte0, e4e6 in byte2
  odd = (odd | (odd >> 4)) & 0x00FF00FFu;
  even = (even | (even >> 8)) & 0x0000FFFFu;  // e0 e2 e4 e6 in nibbles 0..3
  odd = (odd | (odd >> 8)) & 0x0000FFFFu;
  return even | (odd << 16);
}

// ------------------------------------------------------------------ quantiser
// One 32-element block exactly as the reference packer computes it
// (transformer_cuda.rs:554-573): f32 maxNum fold from 0, scale = absmax/7 in f32
// (1.0 for an all-zero block), scale stored RNE as f16, q = clamp(round(v/scale)+8)
// with IEEE division by the f32 scale, half-away-from-zero rounding, Rust's
// saturating `as i32` (NaN -> 0) and wrapping i32 add.
__device__ __forceinline__ int rust_as_i32(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return 2147483647;
  if (x < -2147483648.0f) return (int)0x80000000u;
  return __float2int_rz(x);
}

__device__ __forceinline__ uint16_t quantize_block(const float* v, int len, uint8_t* q) {
  float absmax = 0.0f;
  for (int i = 0; i < len; i++) absmax = fmaxf(absmax, fabsf(v[i]));
  const float scale = (absmax > 0.0f) ? __fdiv_rn(absmax, 7.0f) : 1.0f;
  const uint16_t sbits = __half_as_ushort(__float2half_rn(scale));
#pragma unroll
  for (int i = 0; i < kBlock; i++) {
    const float val = (i < len) ? v[i] : 0.0f;
    const float r = roundf(__fdiv_rn(val, scale));
    const int qw = (int)((unsigned)rust_as_i32(r) + 8u);
    q[i] = (uint8_t)(qw < 0 ? 0 : (qw > 15 ? 15 : qw));
  }
  return sbits;
}

// ------------------------------------------------------------------ dequant
// (q - 8) for the 8 codes of one device word, as 4 exact f16x2 values in
// element order: out[0] = (e0,e1), out[1] = (e2,e3), out[2] = (e4,e5), out[3] = (e6,e7).
// 0x6400 | q is the f16 value 1024 + q; 0x6400 | (q << 4) is 1024 + 16q.
__device__ __forceinline__ void dequant_word_f16x2(uint32_t w, uint32_t out[4]) {
  const uint32_t kMagic = 0x64006400u;
  uint32_t lo0, hi0, lo1, hi1;
  const uint32_t w2 = w >> 8;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(lo0) : "r"(w));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(hi0) : "r"(w));
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(lo1) : "r"(w2));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(hi1) : "r"(w2));
  (void)kMagic;
  const uint32_t k1032 = 0x64086408u;  // f16x2 (1032, 1032)
  const uint32_t k1_16 = 0x2C002C00u;  // f16x2 (1/16, 1/16)
  const uint32_t km72 = 0xD480D480u;   // f16x2 (-72, -72)
  asm("sub.f16x2 %0, %1, %2;" : "=r"(out[0]) : "r"(lo0), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[1]) : "r"(hi0), "r"(k1_16), "r"(km72));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(out[2]) : "r"(lo1), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[3]) : "r"(hi1), "r"(k1_16), "r"(km72));
}

// dequant_word_f16x2 of two words wa (A-fragment row g) and wb (row g + 8),
// written straight into the register order of the two m16n8k16 A fragments
// that consume them: A1 = k pairs (e0,e1) and (e2,e3), A2 = (e4,e5) and
// (e6,e7), each as {row g, row g + 8} for the low and then the high k half.
// Same 18 instructions as two dequant_word_f16x2 calls; the operands need no
// reordering before the MMAs.
__device__ __forceinline__ void dequant_pair_mma(uint32_t wa, uint32_t wb, uint32_t A1[4], uint32_t A2[4]) {
  const uint32_t k1032 = 0x64086408u;  // f16x2 (1032, 1032)
  const uint32_t k1_16 = 0x2C002C00u;  // f16x2 (1/16, 1/16)
  const uint32_t km72 = 0xD480D480u;   // f16x2 (-72, -72)
  const uint32_t wa2 = wa >> 8, wb2 = wb >> 8;
  uint32_t t0, t1, t2, t3, t4, t5, t6, t7;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(t0) : "r"(wa));
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(t1) : "r"(wb));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(t2) : "r"(wa));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(t3) : "r"(wb));
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(t4) : "r"(wa2));
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(t5) : "r"(wb2));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(t6) : "r"(wa2));
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(t7) : "r"(wb2));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(A1[0]) : "r"(t0), "r"(k1032));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(A1[1]) : "r"(t1), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(A1[2]) : "r"(t2), "r"(k1_16), "r"(km72));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(A1[3]) : "r"(t3), "r"(k1_16), "r"(km72));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(A2[0]) : "r"(t4), "r"(k1032));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(A2[1]) : "r"(t5), "r"(k1032));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(A2[2]) : "r"(t6), "r"(k1_16), "r"(km72));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(A2[3]) : "r"(t7), "r"(k1_16), "r"(km72));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// acc += a.x*b.x + a.y*b.y with f16 inputs, exact products, f32 accumulation
// (sm_100 mixed-precision fma).
__device__ __forceinline__ float dot2_f16_f32(uint32_t a, uint32_t b, float acc) {
  uint16_t ax, ay, bx, by;
  asm("mov.b32 {%0, %1}, %2;" : "=h"(ax), "=h"(ay) : "r"(a));
  asm("mov.b32 {%0, %1}, %2;" : "=h"(bx), "=h"(by) : "r"(b));
  asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(ax), "h"(bx));
  asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(ay), "h"(by));
  return acc;
}

// ------------------------------------------------------------------ PDL
// Programmatic dependent launch: the kernels are launched with
// cudaLaunchAttributeProgrammaticStreamSerialization, so they may start while the
// previous kernel in the stream drains.  Everything before grid_dep_wait() must
// not read data the previous kernel writes (weights are safe, activations are not).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t tc_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// Read-only 128-bit load of weight data that is not reused by this SM: bypasses
// L1 allocation; not volatile, so the compiler may batch and reorder it.
__device__ __forceinline__ uint4 ld_weights_u4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------------ shared device helpers
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                                          const uint32_t a3, const uint32_t b0, const uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Output code of the kernels' epilogues (internal, not ABI): bit 0 = f16 output
// (else f32), bit 1 = GELU applied to alpha * acc + bias before the beta term.
constexpr int kOutF16 = 1;
constexpr int kOutGelu = 2;

// GELU, tanh form, as the reference's gelu_fwd states it (lold3344/ARIA
// src/kernels.cu:574-583): 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3)))
// (Hendrycks & Gimpel's approximation).  Evaluated through the identity
// 0.5 (1 + tanh u) = 1 / (1 + exp(-2u)), i.e. v / (1 + exp(-2u)), with the
// hardware exp and divide intrinsics: relative error ~1e-6, far below the one
// f16 rounding of the output, in ~8 instructions inline (an out-of-line
// accurate tanhf made the fused epilogue of a prefill projection 3-4x slower).
// Large negative v: exp -> +inf and the quotient -> 0, as GELU does.
__device__ __forceinline__ float gelu_fast(float v) {
  const float m2u = -1.5957691216f * fmaf(0.044715f * v, v * v, v);  // -2 sqrt(2/pi) (v + 0.044715 v^3)
  return __fdividef(v, 1.0f + __expf(m2u));
}

// Epilogue of CAP outputs of one thread: y[idx(i)] = [GELU](v[i]) + beta *
// y[idx(i)] for the i with ok(i), f16 or f32 (ydt).  idx and ok are functors
// of i; idx(i) must be a valid output index for EVERY i (masked elements point
// at some in-range output, e.g. clamped coordinates).  The old values are then
// loaded unconditionally, all before the first store: a load of y cannot move
// above a store to y (they may alias) and a predicated load feeding a select
// stalls on its result, so a guarded read-modify-write per element serialises
// one memory round trip per output (measured 6x slower on B200; the residual
// add had made a prefill projection up to 9x slower that way).
template <int CAP, class Idx, class Ok>
__device__ __forceinline__ void store_outputs(void* y, int ydt, float (&v)[CAP], float beta, Idx idx, Ok ok) {
  if (ydt & kOutGelu) {
#pragma unroll
    for (int i = 0; i < CAP; i++) v[i] = gelu_fast(v[i]);
  }
  if (ydt & kOutF16) {
    __half* yp = reinterpret_cast<__half*>(y);
    if (beta != 0.0f) {
      __half old[CAP];
#pragma unroll
      for (int i = 0; i < CAP; i++) old[i] = yp[idx(i)];
#pragma unroll
      for (int i = 0; i < CAP; i++) v[i] = fmaf(beta, __half2float(old[i]), v[i]);
    }
#pragma unroll
    for (int i = 0; i < CAP; i++)
      if (ok(i)) yp[idx(i)] = __float2half_rn(v[i]);
  } else {
    float* yp = reinterpret_cast<float*>(y);
    if (beta != 0.0f) {
      float old[CAP];
#pragma unroll
      for (int i = 0; i < CAP; i++) old[i] = yp[idx(i)];
#pragma unroll
      for (int i = 0; i < CAP; i++) v[i] = fmaf(beta, old[i], v[i]);
    }
#pragma unroll
    for (int i = 0; i < CAP; i++)
      if (ok(i)) yp[idx(i)] = v[i];
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(const float* local_addr, uint32_t rank) {
  uint32_t remote, v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(tc_smem_u32(local_addr)), "r"(rank));
  asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(v) : "r"(remote) : "memory");
  return __uint_as_float(v);
}

}  // namespace aria_q4
