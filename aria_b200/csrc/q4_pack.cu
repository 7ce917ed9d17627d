// q4_pack.cu -- bit-exact Q4_0 packer, dequantiser and the loaders that build
// the device-resident tiled form.
//
//   pack_aos_kernel       ARIA quantize_q4_0 (transformer_cuda.rs:549-575) on the
//                         GPU: flat f16/f32 -> 18-byte GGUF blocks, byte-identical.
//   unpack_aos_kernel     the exact inverse (q-8)*scale, for checking and export.
//   repack_{nk,kn}_kernel GGUF blocks -> tiled planes (what a Q4_0 GGUF loader
//                         uploads; the reference's loader reads only f16 tensors,
//                         src/transformer_cuda.rs:3046-3065).
//   quantize_tiled_*      f16 weights -> tiled planes directly, sharing the exact
//                         block quantiser with pack_aos_kernel.
#include "q4_common.cuh"

namespace aria_q4 {

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half* p) { return __half2float(*p); }

// One thread per 32-element block; the CTA's 256 blocks (4608 bytes, 16-byte
// aligned when dst is) are staged in shared memory and written out coalesced.
template <typename T>
__global__ void __launch_bounds__(256) pack_aos_kernel(const T* __restrict__ src, size_t n,
                                                       uint8_t* __restrict__ dst) {
  __shared__ __align__(16) uint8_t stage[256 * kBlockBytes];
  const size_t nblocks = (n + kBlock - 1) / kBlock;
  const size_t b0 = (size_t)blockIdx.x * 256;
  const size_t b = b0 + threadIdx.x;
  if (b < nblocks) {
    float v[kBlock];
    const size_t start = b * kBlock;
    const int len = (int)((n - start) < (size_t)kBlock ? (n - start) : (size_t)kBlock);
    for (int i = 0; i < kBlock; i++) v[i] = (i < len) ? load_as_f32<T>(src + start + i) : 0.0f;
    uint8_t q[kBlock];
    const uint16_t s = quantize_block(v, len, q);
    uint8_t* o = stage + threadIdx.x * kBlockBytes;
    o[0] = (uint8_t)(s & 0xFF);
    o[1] = (uint8_t)(s >> 8);
#pragma unroll
    for (int j = 0; j < 16; j++) o[2 + j] = (uint8_t)(q[2 * j] | (q[2 * j + 1] << 4));
  }
  __syncthreads();
  const size_t nb_here = (nblocks - b0) < 256 ? (nblocks - b0) : 256;
  const size_t bytes = nb_here * kBlockBytes;
  uint8_t* out = dst + b0 * kBlockBytes;
  if (((uintptr_t)out & 15u) == 0) {
    const size_t nvec = bytes / 16;
    for (size_t i = threadIdx.x; i < nvec; i += 256)
      reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(stage)[i];
    for (size_t i = nvec * 16 + threadIdx.x; i < bytes; i += 256) out[i] = stage[i];
  } else {
    for (size_t i = threadIdx.x; i < bytes; i += 256) out[i] = stage[i];
  }
}

__global__ void unpack_aos_kernel(const uint8_t* __restrict__ blocks, size_t n, float* __restrict__ dst) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* blk = blocks + (i / kBlock) * kBlockBytes;
  const float s = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
  const int j = (int)(i % kBlock);
  const uint8_t byte = blk[2 + j / 2];
  const int q = (j & 1) ? (byte >> 4) : (byte & 0xF);
  dst[i] = (float)(q - 8) * s;
}

// NK: one thread per device word.  The 8 codes of word w of row n are 4
// consecutive bytes of one GGUF block of the flat embed[n][k].
__global__ void repack_nk_qs_kernel(const uint8_t* __restrict__ blocks, int K, int N, uint8_t* __restrict__ qs) {
  const int WPR = padded_k(K) / 8;  // words per row
  const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (size_t)N * WPR) return;
  const int n = (int)(id / WPR), w = (int)(id % WPR);
  const int k0 = qs_k_of_word(w);
  uint32_t word = 0x88888888u;  // padding k >= K: code 8, i.e. weight 0
  if (k0 < K) {
    const uint8_t* src = blocks + ((size_t)n * (K / kBlock) + k0 / kBlock) * kBlockBytes + 2 + (k0 % kBlock) / 2;
    const uint32_t r = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) | ((uint32_t)src[3] << 24);
    word = ref_word_to_dev(r);
  }
  reinterpret_cast<uint32_t*>(qs + (size_t)n * qs_row_bytes(K))[w] = word;
}

__global__ void repack_nk_scales_kernel(const uint8_t* __restrict__ blocks, int K, int N, __half* __restrict__ scales) {
  const int BPR = padded_k(K) / kBlock;
  const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (size_t)N * BPR) return;
  const int n = (int)(id / BPR), b = (int)(id % BPR);
  uint16_t s = 0;
  if (b < K / kBlock) {
    const uint8_t* src = blocks + ((size_t)n * (K / kBlock) + b) * kBlockBytes;
    s = (uint16_t)(src[0] | (src[1] << 8));
  }
  scales[((size_t)(b >> 2) * N + n) * 4 + (b & 3)] = __ushort_as_half(s);  // group-major [Kp/128][N][4]
}

// KN: block (k, g) covers n = 32g..32g+31 at row k.  A CTA takes the 128 k-rows
// of one 128-k group G for one 32-column group g, stages the codes in shared
// memory and writes the group's 16 words for each of the 32 device rows.
__device__ __forceinline__ void write_kn_tile(const uint8_t (*codes)[kBlock], int G, int g, int K,
                                              uint8_t* __restrict__ qs) {
  for (int idx = threadIdx.x; idx < 32 * 16; idx += blockDim.x) {
    const int n = idx / 16, w = idx % 16;
    const int kl = qs_k_of_word(w);  // k offset inside the group
    uint8_t q8[8];
#pragma unroll
    for (int i = 0; i < 8; i++) q8[i] = codes[kl + i][n];
    const size_t row = (size_t)g * 32 + n;
    reinterpret_cast<uint32_t*>(qs + row * qs_row_bytes(K))[16 * G + w] = dev_word_from_codes(q8);
  }
}

__global__ void __launch_bounds__(128) repack_kn_kernel(const uint8_t* __restrict__ blocks, int K, int N,
                                                        uint8_t* __restrict__ qs, __half* __restrict__ scales) {
  __shared__ uint8_t codes[128][kBlock];
  const int G32 = N / kBlock;
  const int g = blockIdx.y, G = blockIdx.x;
  const int k = G * 128 + threadIdx.x;
  const int Kp = padded_k(K);
  if (k < K) {
    const uint8_t* src = blocks + ((size_t)k * G32 + g) * kBlockBytes;
    scales[(size_t)g * Kp + k] = __ushort_as_half((uint16_t)(src[0] | (src[1] << 8)));
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const uint8_t byte = src[2 + j];
      codes[threadIdx.x][2 * j] = byte & 0xF;
      codes[threadIdx.x][2 * j + 1] = byte >> 4;
    }
  } else {
    scales[(size_t)g * Kp + k] = __ushort_as_half((uint16_t)0);
#pragma unroll
    for (int j = 0; j < kBlock; j++) codes[threadIdx.x][j] = 8;
  }
  __syncthreads();
  write_kn_tile(codes, G, g, K, qs);
}

// NK: one thread per (row, 32-k block) quantises the block and scatters its four
// device words (word 4t+i of the 128-k group holds the block's k = 8t..8t+7).
template <typename T>
__global__ void quantize_tiled_nk_kernel(const T* __restrict__ w, int K, int N, uint8_t* __restrict__ qs,
                                         __half* __restrict__ scales) {
  const int BPR = padded_k(K) / kBlock;
  const size_t id = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (size_t)N * BPR) return;
  const int n = (int)(id / BPR), b = (int)(id % BPR);
  uint32_t* row = reinterpret_cast<uint32_t*>(qs + (size_t)n * qs_row_bytes(K));
  const int G = b >> 2, i = b & 3;
  const size_t sidx = ((size_t)G * N + n) * 4 + i;  // group-major [Kp/128][N][4]
  if (b * kBlock >= K) {
#pragma unroll
    for (int t = 0; t < 4; t++) row[16 * G + 4 * t + i] = 0x88888888u;
    scales[sidx] = __ushort_as_half((uint16_t)0);
    return;
  }
  float v[kBlock];
  const T* src = w + (size_t)n * K + (size_t)b * kBlock;
#pragma unroll
  for (int e = 0; e < kBlock; e++) v[e] = load_as_f32<T>(src + e);
  uint8_t q[kBlock];
  const uint16_t s = quantize_block(v, kBlock, q);
#pragma unroll
  for (int t = 0; t < 4; t++) row[16 * G + 4 * t + i] = dev_word_from_codes(q + 8 * t);
  scales[sidx] = __ushort_as_half(s);
}

template <typename T>
__global__ void __launch_bounds__(128) quantize_tiled_kn_kernel(const T* __restrict__ w, int K, int N,
                                                                uint8_t* __restrict__ qs,
                                                                __half* __restrict__ scales) {
  __shared__ uint8_t codes[128][kBlock];
  const int g = blockIdx.y, G = blockIdx.x;
  const int k = G * 128 + threadIdx.x;
  const int Kp = padded_k(K);
  if (k < K) {
    float v[kBlock];
    const T* src = w + (size_t)k * N + (size_t)g * kBlock;
#pragma unroll
    for (int i = 0; i < kBlock; i++) v[i] = load_as_f32<T>(src + i);
    uint8_t q[kBlock];
    const uint16_t s = quantize_block(v, kBlock, q);
    scales[(size_t)g * Kp + k] = __ushort_as_half(s);
#pragma unroll
    for (int i = 0; i < kBlock; i++) codes[threadIdx.x][i] = q[i];
  } else {
    scales[(size_t)g * Kp + k] = __ushort_as_half((uint16_t)0);
#pragma unroll
    for (int i = 0; i < kBlock; i++) codes[threadIdx.x][i] = 8;
  }
  __syncthreads();
  write_kn_tile(codes, G, g, K, qs);
}

// ------------------------------------------------------------------ launchers

cudaError_t launch_pack_f16(const uint16_t* src, size_t n, uint8_t* dst, cudaStream_t st) {
  const size_t nb = (n + kBlock - 1) / kBlock;
  if (nb == 0) return cudaSuccess;
  pack_aos_kernel<__half><<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(reinterpret_cast<const __half*>(src), n, dst);
  return cudaGetLastError();
}

cudaError_t launch_pack_f32(const float* src, size_t n, uint8_t* dst, cudaStream_t st) {
  const size_t nb = (n + kBlock - 1) / kBlock;
  if (nb == 0) return cudaSuccess;
  pack_aos_kernel<float><<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(src, n, dst);
  return cudaGetLastError();
}

cudaError_t launch_unpack(const uint8_t* blocks, size_t n, float* dst, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  unpack_aos_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(blocks, n, dst);
  return cudaGetLastError();
}

cudaError_t launch_repack(const uint8_t* blocks, int layout, int K, int N, uint8_t* tiled, cudaStream_t st) {
  uint8_t* qs = tiled;
  __half* scales = reinterpret_cast<__half*>(tiled + tiled_scale_offset(K, N));
  const int Kp = padded_k(K);
  if (layout == 1) {
    const size_t nw = (size_t)N * (Kp / 8);
    repack_nk_qs_kernel<<<(unsigned)((nw + 255) / 256), 256, 0, st>>>(blocks, K, N, qs);
    const size_t nb = (size_t)N * (Kp / kBlock);
    repack_nk_scales_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, st>>>(blocks, K, N, scales);
  } else {
    dim3 grid(Kp / 128, N / kBlock);
    repack_kn_kernel<<<grid, 128, 0, st>>>(blocks, K, N, qs, scales);
  }
  return cudaGetLastError();
}

cudaError_t launch_quantize_tiled(const uint16_t* w, int layout, int K, int N, uint8_t* tiled, cudaStream_t st) {
  uint8_t* qs = tiled;
  __half* scales = reinterpret_cast<__half*>(tiled + tiled_scale_offset(K, N));
  const __half* wh = reinterpret_cast<const __half*>(w);
  const int Kp = padded_k(K);
  if (layout == 1) {
    const size_t nb = (size_t)N * (Kp / kBlock);
    quantize_tiled_nk_kernel<__half><<<(unsigned)((nb + 127) / 128), 128, 0, st>>>(wh, K, N, qs, scales);
  } else {
    dim3 grid(Kp / 128, N / kBlock);
    quantize_tiled_kn_kernel<__half><<<grid, 128, 0, st>>>(wh, K, N, qs, scales);
  }
  return cudaGetLastError();
}

}  // namespace aria_q4
