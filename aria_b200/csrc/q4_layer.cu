// q4_layer.cu -- the non-projection work of one decode step on the GPU.
//
// ARIA decodes with KV cache only on the CPU (lold3344/ARIA
// src/transformer_cuda.rs `step` :1286-1324 over `cpu_layer_forward`
// :1059-1166); its GPU forward recomputes the whole prompt every token.  With
// the Q4_0 projections on the GPU, the rest of a decode step is three small
// kernels, all stream-ordered and allocation-free:
//
//  * embed_kernel      h[m] = embed[token_m] + pos_embed[pos_m]        (:1294-1297)
//  * layernorm_kernel  y[m] = (x[m] - mean) * rstd * g + b, eps 1e-5    (cpu_layernorm :3271-3293)
//  * attention_kernel  one new token per sequence: append its k, v to the
//                      cache at pos_m, then per head softmax(q.K^T / sqrt(dh))
//                      over positions 0..pos_m and the weighted sum of V
//                      (:1098-1137; causal: the new token sees itself and
//                      the cache)
//
// The residual stream h stays f32 (the projections add into it through their
// beta = 1 epilogue); LayerNorm, attention and the KV cache store f16, the
// activation type the projections read.  One CTA per sequence row (LayerNorm)
// or per (sequence, head) (attention): these kernels touch kilobytes per token
// and are latency-bound, not bandwidth-bound.
#include "q4_common.cuh"

namespace aria_q4 {

constexpr int kLayerThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
  for (int w = 0; w < nw; w++) s += red[w];
  return s;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = -INFINITY;
  for (int w = 0; w < nw; w++) s = fmaxf(s, red[w]);
  return s;
}

// h[m][j] = embed[tok[m]][j] + pos_embed[pos[m]][j] (f16 tables, f32 out);
// token and position clamped into the tables as the reference clamps them
// (`tok.min(vocab_size - 1)`, `pos.min(max_seq_len - 1)`, :1291-1292)
__global__ void __launch_bounds__(kLayerThreads) embed_kernel(const __half* embed, const __half* pos_embed,
                                                              const int* tok, const int* pos, int vocab, int max_seq,
                                                              int d, float* h) {
  grid_dep_launch();  // the next projection (programmatic dependence) may load its weights meanwhile
  const int m = blockIdx.x;
  const int tk = min(max(tok[m], 0), vocab - 1), ps = min(max(pos[m], 0), max_seq - 1);
  const __half* e = embed + (size_t)tk * d;
  const __half* p = pos_embed + (size_t)ps * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) h[(size_t)m * d + j] = __half2float(e[j]) + __half2float(p[j]);
}

// y[m] = (x[m] - mean) * rstd * g + b over d f32 values, f16 out.  Two passes
// over the row held in registers (mean, then the centred variance), like the
// reference's f32 LayerNorm.
template <int PER>  // values per thread: d <= PER * kLayerThreads
__global__ void __launch_bounds__(kLayerThreads) layernorm_kernel(const float* x, const __half* g, const __half* b,
                                                                  int d, float eps, __half* y, int ldy) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const float* xr = x + (size_t)m * d;
  float v[PER];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int j = threadIdx.x + i * kLayerThreads;
    v[i] = j < d ? xr[j] : 0.0f;
    s += v[i];
  }
  const float mean = block_sum(s, red) / (float)d;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int j = threadIdx.x + i * kLayerThreads;
    const float c = j < d ? v[i] - mean : 0.0f;
    q = fmaf(c, c, q);
  }
  const float var = block_sum(q, red) / (float)d;
  const float rs = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int j = threadIdx.x + i * kLayerThreads;
    if (j < d) y[(size_t)m * ldy + j] = __float2half_rn((v[i] - mean) * rs * __half2float(g[j]) + __half2float(b[j]));
  }
}

// One CTA per (sequence m, head hd), head dimension DH.  qkv [M][3d] f16 holds
// this token's q, k, v; the caches are f16 [M][max_seq][d].  The token's own
// k, v are read from the qkv row and stored at pos[m] in the caches (for the
// following steps); positions 0..pos-1 come from the caches.  Nothing waits
// on that store, so the dependent loads are: the position, then every K row
// (a thread per position, DH/8 16-byte loads issued before the first
// multiply; the V rows are prefetched into L2 at the same time), then the V
// values.  Scores are softmaxed in f32 (max-subtracted) in shared memory and
// the weighted sum of V is formed by (head dimension pair, position group)
// threads, 16 positions' values loaded before their multiply-adds.  scores:
// shared memory of max_seq floats.
template <int DH>
__global__ void __launch_bounds__(kLayerThreads) attention_kernel(const __half* qkv, int d, int max_seq,
                                                                  const int* pos, __half* kc, __half* vc,
                                                                  __half* out, float scale) {
  extern __shared__ float sm[];  // [max_seq] scores, [DH] q, [2 kLayerThreads] partial sums
  float* sc = sm;
  float* qs = sm + max_seq;
  float* part = qs + DH;
  __shared__ float red[32];
  const int m = blockIdx.x, hd = blockIdx.y, tid = threadIdx.x;
  const __half* row = qkv + (size_t)m * 3 * d;
  const __half* qn = row + hd * DH;          // this token's q, k, v for the head
  const __half* kn = row + d + hd * DH;
  const __half* vn = row + 2 * d + hd * DH;
  __half qe = __float2half_rn(0.0f), ke = qe, ve = qe;
  if (tid < DH) {  // DH <= kLayerThreads: one element each, loaded alongside the position
    qe = qn[tid];
    ke = kn[tid];
    ve = vn[tid];
  }
  const int p = pos[m];
  if (p < 0 || p >= max_seq) {  // no cache slot: the caller's position is out of range
    for (int j = tid; j < DH; j += blockDim.x) out[(size_t)m * d + hd * DH + j] = __float2half_rn(0.0f);
    return;
  }
  __half* kcm = kc + (size_t)m * max_seq * d + hd * DH;
  __half* vcm = vc + (size_t)m * max_seq * d + hd * DH;
  const int n = p + 1;
  auto krow = [&](int i) -> const uint4* {
    return reinterpret_cast<const uint4*>(i == p ? kn : kcm + (size_t)i * d);
  };
  // first position of this thread: its K row in flight before anything else
  uint4 kw[DH / 8];
  if (tid < n) {
    const uint4* kr = krow(tid);
#pragma unroll
    for (int j = 0; j < DH / 8; j++) kw[j] = kr[j];
  }
  for (int i = tid; i < p; i += blockDim.x) bulk_prefetch_l2(vcm + (size_t)i * d, DH * 2);
  if (tid < DH) {
    qs[tid] = __half2float(qe);
    kcm[(size_t)p * d + tid] = ke;
    vcm[(size_t)p * d + tid] = ve;
  }
  __syncthreads();  // qs
  float mx = -INFINITY;
  for (int i = tid; i < n; i += blockDim.x) {
    if (i != tid) {
      const uint4* kr = krow(i);
#pragma unroll
      for (int j = 0; j < DH / 8; j++) kw[j] = kr[j];
    }
    float dot = 0.0f;
#pragma unroll
    for (int j = 0; j < DH / 8; j++) {
      const uint32_t ws[4] = {kw[j].x, kw[j].y, kw[j].z, kw[j].w};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float2 kv = __half22float2(*reinterpret_cast<const __half2*>(&ws[u]));
        dot = fmaf(qs[8 * j + 2 * u], kv.x, dot);
        dot = fmaf(qs[8 * j + 2 * u + 1], kv.y, dot);
      }
    }
    const float s = dot * scale;
    sc[i] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_max(mx, red);
  float sum = 0.0f;
  for (int i = tid; i < n; i += blockDim.x) {
    const float e = __expf(sc[i] - mx);
    sc[i] = e;
    sum += e;
  }
  sum = block_sum(sum, red);  // its barriers also publish sc[]
  // the scores are done: let the next kernel (attn_out, launched with
  // programmatic dependence) start loading its weights while the weighted sum
  // of V runs; it still waits for this grid to complete before reading out
  grid_dep_launch();
  const float inv = 1.0f / sum;
  // weighted sum of V: thread = (dimension pair jp, position group pg); up to
  // 16 positions' pairs loaded before their multiply-adds
  constexpr int kPairs = DH / 2, kGroups = kLayerThreads / kPairs;
  const int jp = tid % kPairs, pg = tid / kPairs;
  auto vrow = [&](int i) -> const __half* { return i == p ? vn : vcm + (size_t)i * d; };
  float ax = 0.0f, ay = 0.0f;
  int i = pg;
  for (; i + 15 * kGroups < n; i += 16 * kGroups) {
    __half2 v[16];
#pragma unroll
    for (int u = 0; u < 16; u++) v[u] = *reinterpret_cast<const __half2*>(vrow(i + u * kGroups) + 2 * jp);
#pragma unroll
    for (int u = 0; u < 16; u++) {
      const float2 f = __half22float2(v[u]);
      const float w = sc[i + u * kGroups];
      ax = fmaf(w, f.x, ax);
      ay = fmaf(w, f.y, ay);
    }
  }
  for (; i < n; i += kGroups) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vrow(i) + 2 * jp));
    ax = fmaf(sc[i], f.x, ax);
    ay = fmaf(sc[i], f.y, ay);
  }
  part[2 * tid] = ax;
  part[2 * tid + 1] = ay;
  __syncthreads();
  if (tid < kPairs) {
    float ox = 0.0f, oy = 0.0f;
#pragma unroll
    for (int g2 = 0; g2 < kGroups; g2++) {
      ox += part[2 * (g2 * kPairs + tid)];
      oy += part[2 * (g2 * kPairs + tid) + 1];
    }
    *reinterpret_cast<__half2*>(out + (size_t)m * d + hd * DH + 2 * tid) = __floats2half2_rn(ox * inv, oy * inv);
  }
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_embed(const __half* embed, const __half* pos_embed, const int* tok, const int* pos, int M, int vocab,
                         int max_seq, int d, float* h, cudaStream_t st) {
  embed_kernel<<<M, kLayerThreads, 0, st>>>(embed, pos_embed, tok, pos, vocab, max_seq, d, h);
  return cudaGetLastError();
}

// The same LayerNorm with one warp per row (rows of d <= 128 V4 values, d a
// multiple of 4): 16-byte loads of x, 8-byte loads of g, b and stores of y,
// the row held in registers, warp-shuffle sums.  Eight rows per CTA.  For the
// whole-prompt forward's [tokens][896] rows it moves ~2.5x the bytes per
// second of the CTA-per-row kernel, which spends most of its time in block
// barriers on rows this short.
template <int V4>
__global__ void __launch_bounds__(kLayerThreads) layernorm_warp_kernel(const float* x, const __half* g,
                                                                       const __half* b, int M, int d, float eps,
                                                                       __half* y, int ldy) {
  grid_dep_launch();  // the next projection (programmatic dependence) may load its weights meanwhile
  const int row = (int)blockIdx.x * (kLayerThreads / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const int n4 = d >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * d);
  float4 v[V4];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < V4; i++) {
    const int j = lane + 32 * i;
    v[i] = j < n4 ? xr[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)d;
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < V4; i++) {
    if (lane + 32 * i < n4) {
      const float c0 = v[i].x - mean, c1 = v[i].y - mean, c2 = v[i].z - mean, c3 = v[i].w - mean;
      q = fmaf(c0, c0, q);
      q = fmaf(c1, c1, q);
      q = fmaf(c2, c2, q);
      q = fmaf(c3, c3, q);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rs = rsqrtf(q / (float)d + eps);
  __half* yr = y + (size_t)row * ldy;
#pragma unroll
  for (int i = 0; i < V4; i++) {
    const int j = lane + 32 * i;
    if (j < n4) {
      const uint2 gw = reinterpret_cast<const uint2*>(g)[j];
      const uint2 bw = reinterpret_cast<const uint2*>(b)[j];
      const float2 g01 = __half22float2(*reinterpret_cast<const __half2*>(&gw.x));
      const float2 g23 = __half22float2(*reinterpret_cast<const __half2*>(&gw.y));
      const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&bw.x));
      const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&bw.y));
      const __half2 o01 = __floats2half2_rn((v[i].x - mean) * rs * g01.x + b01.x, (v[i].y - mean) * rs * g01.y + b01.y);
      const __half2 o23 = __floats2half2_rn((v[i].z - mean) * rs * g23.x + b23.x, (v[i].w - mean) * rs * g23.y + b23.y);
      uint2 ow;
      ow.x = *reinterpret_cast<const uint32_t*>(&o01);
      ow.y = *reinterpret_cast<const uint32_t*>(&o23);
      reinterpret_cast<uint2*>(yr)[j] = ow;
    }
  }
}

cudaError_t launch_layernorm(const float* x, const __half* g, const __half* b, int M, int d, float eps, __half* y,
                             int ldy, cudaStream_t st) {
  const bool vec = d % 4 == 0 && d <= 1024 && ldy % 4 == 0 && ((uintptr_t)x & 15u) == 0 &&
                   ((uintptr_t)g & 7u) == 0 && ((uintptr_t)b & 7u) == 0 && ((uintptr_t)y & 7u) == 0;
  if (vec) {
    const int rows_per_cta = kLayerThreads / 32;
    const int grid = (M + rows_per_cta - 1) / rows_per_cta;
    if (d <= 512)
      layernorm_warp_kernel<4><<<grid, kLayerThreads, 0, st>>>(x, g, b, M, d, eps, y, ldy);
    else
      layernorm_warp_kernel<8><<<grid, kLayerThreads, 0, st>>>(x, g, b, M, d, eps, y, ldy);
    return cudaGetLastError();
  }
  const int per = (d + kLayerThreads - 1) / kLayerThreads;
  if (per <= 4) layernorm_kernel<4><<<M, kLayerThreads, 0, st>>>(x, g, b, d, eps, y, ldy);
  else if (per <= 16) layernorm_kernel<16><<<M, kLayerThreads, 0, st>>>(x, g, b, d, eps, y, ldy);
  else layernorm_kernel<32><<<M, kLayerThreads, 0, st>>>(x, g, b, d, eps, y, ldy);
  return cudaGetLastError();
}

size_t attention_smem_bytes(int dh, int max_seq) { return (size_t)(max_seq + dh + 2 * kLayerThreads) * sizeof(float); }

cudaError_t launch_attention(const __half* qkv, int M, int d, int heads, int max_seq, const int* pos, __half* kc,
                             __half* vc, __half* out, cudaStream_t st) {
  const int dh = d / heads;
  const size_t smem = attention_smem_bytes(dh, max_seq);
  const float scale = 1.0f / sqrtf((float)dh);
  auto run = [&](auto kern) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    kern<<<dim3(M, heads), kLayerThreads, smem, st>>>(qkv, d, max_seq, pos, kc, vc, out, scale);
    return cudaGetLastError();
  };
  switch (dh) {
    case 32: return run(attention_kernel<32>);
    case 64: return run(attention_kernel<64>);
    case 128: return run(attention_kernel<128>);
    case 256: return run(attention_kernel<256>);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace aria_q4
