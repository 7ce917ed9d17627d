// q4_decode.cu -- decode / skinny regime Q4_0 projection (M <= 32 token rows).
//
// Replaces, for Q4_0 weights, the cuBLAS fp16 GEMM that ARIA runs for every
// projection (`gemm()` at lold3344/ARIA src/transformer_cuda.rs:615-640, called
// at :1583 QKV, :1686 attn_out, :1753 ffn_up, :1805 ffn_down, :1864 LM head).
// At M <= 32 that product is bound by weight bytes: this kernel streams 0.5625 B
// per weight (the Q4_0 codes and scales) instead of the 2 B of f16 weights.
//
// Design (B200): the weights never touch shared memory.  A warp owns a tile of
// 16 output rows and a K-slice; each lane issues one 128-bit load per row pair
// per 128 k (the tiled layout puts a lane's 8-k slice of four 32-k blocks in 16
// contiguous bytes), turns the codes into exact (q-8) f16x2 values with
// LOP3/HSUB (9 instructions per 8 weights), and feeds them as the A fragment of
// warp-level m16n8k16 tensor-core MMAs with f32 accumulation; the activations
// are the B fragment (k is permuted consistently on both sides, so lane t's
// fragment is k = 8t..8t+7 of each 32-k block).  A SIMT dot product with the
// same dequantisation needs about 4x more issue slots per weight and measured
// issue-bound at ~2 TB/s on B200; the tensor-core form leaves the kernel
// HBM-bound.  tcgen05 is not used here: at M <= 32 the MMA is not the
// bottleneck, and staging dequantised weights through shared memory for
// tcgen05 would cost 4 B of shared-memory traffic per weight.
//
// Scales: NK (blocks along k) -- one scale per (row, 32-k block), stored
// group-major so a row pair's four block scales are one 8-byte load; the block's two
// MMAs accumulate from zero and are scaled in f32: exact products, f32 sums.
// KN (blocks along n) -- one scale per (k, 32-row group); it is folded into the
// activation fragment (x*s rounded to f16, relative error <= 2^-11).
//
// K is split across the warps of a CTA (up to 8); partial fragments are reduced
// in shared memory.  No global scratch.  Launch uses programmatic dependent
// launch: before griddepcontrol.wait a CTA only prefetches its weight rows to
// L2, so weight streaming overlaps the previous kernel's tail.
#include "q4_common.cuh"

namespace aria_q4 {

struct DecodeArgs {
  const uint8_t* qs;
  const __half* scales;
  int K, N, Kp;
  const __half* x;
  int ldx, M;
  void* y;
  int ydt, ldy;
  const __half* bias;
  float alpha, beta;
  int ksplit;  // warps per 16-row tile
};

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

__device__ __forceinline__ void store_out(void* y, int ydt, size_t idx, float v, float beta) {
  if (ydt == 0) {
    float* yp = reinterpret_cast<float*>(y) + idx;
    if (beta != 0.0f) v += beta * *yp;
    *yp = v;
  } else {
    __half* yp = reinterpret_cast<__half*>(y) + idx;
    if (beta != 0.0f) v += beta * __half2float(*yp);
    *yp = __float2half_rn(v);
  }
}

__device__ __forceinline__ uint4 ld_u4_or(const void* p, bool ok, uint32_t fill) {
  return ok ? ld_weights_u4(p) : make_uint4(fill, fill, fill, fill);
}

// One 128-k group of a 16-row tile for one warp: 2 rows x 16 bytes per lane.
struct GroupRegs {
  uint4 qa, qb;
  uint2 sa, sb;
};

template <int LAYOUT, int NT, int MAXB>
__global__ void __launch_bounds__(256, 2) decode_mma_kernel(const DecodeArgs a) {
  __shared__ float red[8][32][NT * 4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int S = a.ksplit;
  const int tiles_per_cta = 8 / S;
  const int slot = warp / S, ks = warp % S;
  const bool active_warp = slot < tiles_per_cta;
  const int tile = blockIdx.x * tiles_per_cta + slot;
  const int r0 = tile * 16;
  const int KG = a.Kp >> 7;
  const int gps = (KG + S - 1) / S;
  const int gbeg = ks * gps, gend = min(KG, gbeg + gps);
  const size_t RB = (size_t)a.Kp >> 1;
  const int m0 = blockIdx.y * 8 * NT;

  const int ra = r0 + g, rb = r0 + g + 8;
  const bool oka = active_warp && ra < a.N, okb = active_warp && rb < a.N;
  const uint8_t* qa_ptr = a.qs + (size_t)ra * RB + 16 * t;
  const uint8_t* qb_ptr = a.qs + (size_t)rb * RB + 16 * t;

  // weights are load-time constants: start streaming them towards L2 now
  if (active_warp && t == 0 && gend > gbeg) {
    if (oka) bulk_prefetch_l2(a.qs + (size_t)ra * RB + (size_t)gbeg * 64, (uint32_t)(gend - gbeg) * 64u);
    if (okb) bulk_prefetch_l2(a.qs + (size_t)rb * RB + (size_t)gbeg * 64, (uint32_t)(gend - gbeg) * 64u);
  }
  grid_dep_launch();
  grid_dep_wait();

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[j][e] = 0.0f;

  const int grp = r0 >> 5;   // 32-row scale group (KN)

  if (active_warp) {
    for (int gb = gbeg; gb < gend; gb += MAXB) {
      const int nb = min(MAXB, gend - gb);
      // issue every load of this batch before any arithmetic (up to MAXB KB in flight per warp)
      GroupRegs R[MAXB];
#pragma unroll
      for (int u = 0; u < MAXB; u++) {
        if (u < nb) {
          const int G = gb + u;
          R[u].qa = ld_u4_or(qa_ptr + (size_t)G * 64, oka, 0x88888888u);
          R[u].qb = ld_u4_or(qb_ptr + (size_t)G * 64, okb, 0x88888888u);
          R[u].sa = make_uint2(0, 0);
          R[u].sb = make_uint2(0, 0);
          if (LAYOUT == 1) {
            if (oka) R[u].sa = __ldg(reinterpret_cast<const uint2*>(a.scales + ((size_t)G * a.N + ra) * 4));
            if (okb) R[u].sb = __ldg(reinterpret_cast<const uint2*>(a.scales + ((size_t)G * a.N + rb) * 4));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < MAXB; u++) {
        if (u >= nb) break;
        const int G = gb + u;
        const uint32_t qaw[4] = {R[u].qa.x, R[u].qa.y, R[u].qa.z, R[u].qa.w};
        const uint32_t qbw[4] = {R[u].qb.x, R[u].qb.y, R[u].qb.z, R[u].qb.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int kb = G * 128 + i * 32;
          if (kb >= a.K) break;  // padded tail of K (uniform across the warp)
          uint4 xv[NT];
#pragma unroll
          for (int j = 0; j < NT; j++) {
            const int tok = m0 + 8 * j + g;
            xv[j] = (tok < a.M) ? __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)tok * a.ldx + kb + 8 * t))
                                : make_uint4(0, 0, 0, 0);
          }
          if (LAYOUT == 0) {
            const uint4 s8 = __ldg(reinterpret_cast<const uint4*>(a.scales + (size_t)grp * a.Kp + kb + 8 * t));
#pragma unroll
            for (int j = 0; j < NT; j++) {
              xv[j].x = hmul2_u32(xv[j].x, s8.x);
              xv[j].y = hmul2_u32(xv[j].y, s8.y);
              xv[j].z = hmul2_u32(xv[j].z, s8.z);
              xv[j].w = hmul2_u32(xv[j].w, s8.w);
            }
          }
          uint32_t pa[4], pb[4];
          dequant_word_f16x2(qaw[i], pa);
          dequant_word_f16x2(qbw[i], pb);
#pragma unroll
          for (int j = 0; j < NT; j++) {
            if (LAYOUT == 1) {
              float c[4] = {0.f, 0.f, 0.f, 0.f};
              mma_16816(c, pa[0], pb[0], pa[1], pb[1], xv[j].x, xv[j].y);
              mma_16816(c, pa[2], pb[2], pa[3], pb[3], xv[j].z, xv[j].w);
              const uint32_t swa = (i < 2) ? R[u].sa.x : R[u].sa.y, swb = (i < 2) ? R[u].sb.x : R[u].sb.y;
              const float fa = __half2float(__ushort_as_half((uint16_t)((i & 1) ? (swa >> 16) : (swa & 0xFFFF))));
              const float fb = __half2float(__ushort_as_half((uint16_t)((i & 1) ? (swb >> 16) : (swb & 0xFFFF))));
              acc[j][0] = fmaf(fa, c[0], acc[j][0]);
              acc[j][1] = fmaf(fa, c[1], acc[j][1]);
              acc[j][2] = fmaf(fb, c[2], acc[j][2]);
              acc[j][3] = fmaf(fb, c[3], acc[j][3]);
            } else {
              mma_16816(acc[j], pa[0], pb[0], pa[1], pb[1], xv[j].x, xv[j].y);
              mma_16816(acc[j], pa[2], pb[2], pa[3], pb[3], xv[j].z, xv[j].w);
            }
          }
        }
      }
    }
  }

  if (S > 1) {
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) red[warp][lane][j * 4 + e] = acc[j][e];
    __syncthreads();
    if (ks != 0 || !active_warp) return;
    for (int s = 1; s < S; s++)
#pragma unroll
      for (int j = 0; j < NT; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[j][e] += red[warp + s][lane][j * 4 + e];
  }
  if (!active_warp) return;

  // D fragment: c0,c1 -> (row g, tokens 2t, 2t+1); c2,c3 -> (row g+8, same tokens)
  float bia = 0.f, bib = 0.f;
  if (a.bias) {
    if (oka) bia = __half2float(a.bias[ra]);
    if (okb) bib = __half2float(a.bias[rb]);
  }
#pragma unroll
  for (int j = 0; j < NT; j++) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int tok = m0 + 8 * j + 2 * t + (e & 1);
      const bool rowb = e >= 2;
      const int n = rowb ? rb : ra;
      if (tok < a.M && (rowb ? okb : oka)) {
        const float v = a.alpha * acc[j][e] + (rowb ? bib : bia);
        store_out(a.y, a.ydt, (size_t)tok * a.ldy + n, v, a.beta);
      }
    }
  }
}

template <int LAYOUT, int NT, int MAXB>
static cudaError_t launch_t(const DecodeArgs& a, cudaStream_t st, bool pdl) {
  const int tiles = (a.N + 15) / 16;
  const int tpc = 8 / a.ksplit;
  dim3 grid((tiles + tpc - 1) / tpc, (a.M + 8 * NT - 1) / (8 * NT));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, decode_mma_kernel<LAYOUT, NT, MAXB>, a);
}

template <int LAYOUT, int NT>
static cudaError_t launch_nt(const DecodeArgs& a, int maxb, cudaStream_t st, bool pdl) {
  if (maxb <= 1) return launch_t<LAYOUT, NT, 1>(a, st, pdl);
  if (maxb <= 2) return launch_t<LAYOUT, NT, 2>(a, st, pdl);
  return launch_t<LAYOUT, NT, 4>(a, st, pdl);
}

// Decode-regime projection for M <= 32 (larger M goes to the tcgen05 kernel).
// Work split: a 16-row tile's K is cut into `ksplit` slices (one warp each) only
// when there are too few tiles to give every SM eight warps; a warp then loads
// its whole slice (up to 8 groups = 8 KB per warp) before computing.
cudaError_t launch_decode(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                          int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl) {
  DecodeArgs a;
  a.qs = tiled;
  a.scales = reinterpret_cast<const __half*>(tiled + tiled_scale_offset(K, N));
  a.K = K; a.N = N; a.Kp = padded_k(K);
  a.x = x; a.ldx = ldx; a.M = M; a.y = y; a.ydt = ydt; a.ldy = ldy;
  a.bias = bias; a.alpha = alpha; a.beta = beta;
  const int KG = a.Kp / 128;
  const int tiles = (N + 15) / 16;
  // K-split: enough warps for ~16 per SM, and at most 4 groups (4 KB) per warp
  int S = 1;
  while (S < 8 && S < KG && ((long long)tiles * S < 148LL * 16 || (KG + S - 1) / S > 4)) S++;
  a.ksplit = S;
  const int gpw = (KG + S - 1) / S;
  const int nt = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  if (layout == 1) {
    if (nt == 1) return launch_nt<1, 1>(a, gpw, st, pdl);
    if (nt == 2) return launch_nt<1, 2>(a, gpw, st, pdl);
    return launch_nt<1, 4>(a, gpw, st, pdl);
  }
  if (nt == 1) return launch_nt<0, 1>(a, gpw, st, pdl);
  if (nt == 2) return launch_nt<0, 2>(a, gpw, st, pdl);
  return launch_nt<0, 4>(a, gpw, st, pdl);
}

}  // namespace aria_q4
