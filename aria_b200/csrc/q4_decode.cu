// q4_decode.cu -- decode / skinny regime Q4_0 projection (M <= 64 token rows).
//
// Replaces, for Q4_0 weights, the cuBLAS fp16 GEMM that ARIA runs for every
// projection (`gemm()` at lold3344/ARIA src/transformer_cuda.rs:615-640, called
// at :1583 QKV, :1686 attn_out, :1753 ffn_up, :1805 ffn_down, :1864 LM head).
// At small M that product is bound by weight bytes: this kernel streams 0.5625 B
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
// K is split across the warps of a CTA (up to 8) and, for tall-K shapes with few
// tiles, across a thread-block cluster of up to 4 CTAs; partial fragments are
// reduced in shared memory and then through distributed shared memory.  No
// global scratch.  Launch uses programmatic dependent
// launch: before griddepcontrol.wait a CTA only prefetches its weight rows to
// L2 -- or, when the caller declares the weights constant (not written by the
// preceding kernel), loads its first batch of codes and scales into registers
// -- so weight streaming overlaps the previous kernel's tail.
#include "q4_common.cuh"

namespace aria_q4 {

// row tiles (16 outputs each) at or below which 16-token passes are used
constexpr int kDecodeFewTiles = 64;

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
  int ksplit;  // warps per 16-row tile (within a CTA)
  int csplit;  // CTAs per tile group (a thread-block cluster along x)
  int const_weights;  // weights are not written by the preceding kernel: load them before the dependency wait
  // LayerNorm prologue (h != nullptr): x = LayerNorm(h) rounded to f16, with h
  // f32 [M][ldx], per-k gain / shift ln_g, ln_b (f16 [K]) and ln_eps; x unused
  const float* h;
  const __half* ln_g;
  const __half* ln_b;
  float ln_eps;
};

__device__ __forceinline__ uint4 ld_u4_or(const void* p, bool ok, uint32_t fill) {
  return ok ? ld_weights_u4(p) : make_uint4(fill, fill, fill, fill);
}

// One 128-k group of a 16-row tile for one warp: two rows' codes (16 B per lane),
// NK block scales, and -- when the batch preloads them -- the activation and KN
// scale fragments of the group's four 32-k blocks.
template <int NT, bool PRE>
struct GroupRegs {
  uint4 qa, qb;
  uint2 sa, sb;
  uint4 xv[PRE ? 4 : 1][PRE ? NT : 1];
  uint4 ks[PRE ? 4 : 1];
};

// PRE: the batch phase also loads every activation / KN-scale fragment of its
// groups (small NT), so no load latency is exposed inside the MMA loop.
// LN: the LayerNorm prologue (a separate instance, so that the plain kernel
// keeps its register budget).
template <int LAYOUT, int NT, int MAXB, bool PRE, bool LN>
__global__ void __launch_bounds__(256, 2) decode_mma_kernel(const DecodeArgs a) {
  __shared__ float red[8][32][NT * 4];
  __shared__ float2 ln_stat[8 * NT];  // LayerNorm prologue: (mean, rstd) of this CTA's token rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int S = a.ksplit, C = a.csplit;
  const int tiles_per_cta = 8 / S;
  const int slot = warp / S, ks = warp % S;
  const bool active_warp = slot < tiles_per_cta;
  const int crank = (int)blockIdx.x % C;  // rank in the cluster (clusters run along x)
  const int tile = ((int)blockIdx.x / C) * tiles_per_cta + slot;
  const int r0 = tile * 16;
  const int KG = a.Kp >> 7;
  const int nslices = S * C;
  const int gps = (KG + nslices - 1) / nslices;
  const int gbeg = (crank * S + ks) * gps, gend = min(KG, gbeg + gps);
  const size_t RB = (size_t)a.Kp >> 1;
  const int m0 = blockIdx.y * 8 * NT;

  const int ra = r0 + g, rb = r0 + g + 8;
  const bool oka = active_warp && ra < a.N, okb = active_warp && rb < a.N;
  const uint8_t* qa_ptr = a.qs + (size_t)ra * RB + 16 * t;
  const uint8_t* qb_ptr = a.qs + (size_t)rb * RB + 16 * t;

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[j][e] = 0.0f;

  const int grp = r0 >> 5;  // 32-row scale group (KN)
  auto load_x = [&](int kb, int j) -> uint4 {
    const int tok = m0 + 8 * j + g;
    if (tok >= a.M || kb >= a.K) return make_uint4(0, 0, 0, 0);
    if (!LN) return __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)tok * a.ldx + kb + 8 * t));
    // LayerNorm of the f32 row, (v - mean) * rstd * g + b as the LayerNorm
    // kernel computes it, rounded to f16 as that kernel would store it
    const float* hp = a.h + (size_t)tok * a.ldx + kb + 8 * t;
    const float4 h0 = __ldg(reinterpret_cast<const float4*>(hp));
    const float4 h1 = __ldg(reinterpret_cast<const float4*>(hp + 4));
    const uint4 gw = __ldg(reinterpret_cast<const uint4*>(a.ln_g + kb + 8 * t));
    const uint4 bw = __ldg(reinterpret_cast<const uint4*>(a.ln_b + kb + 8 * t));
    const float2 st = ln_stat[tok - m0];
    const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint32_t gs[4] = {gw.x, gw.y, gw.z, gw.w}, bs[4] = {bw.x, bw.y, bw.z, bw.w};
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float2 gf = __half22float2(*reinterpret_cast<const __half2*>(&gs[u]));
      const float2 bf = __half22float2(*reinterpret_cast<const __half2*>(&bs[u]));
      const __half2 r = __floats2half2_rn((hv[2 * u] - st.x) * st.y * gf.x + bf.x,
                                          (hv[2 * u + 1] - st.x) * st.y * gf.y + bf.y);
      o[u] = *reinterpret_cast<const uint32_t*>(&r);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  auto load_ks = [&](int kb) -> uint4 {
    return (active_warp && kb < a.Kp) ? __ldg(reinterpret_cast<const uint4*>(a.scales + (size_t)grp * a.Kp + kb + 8 * t))
                                      : make_uint4(0, 0, 0, 0);
  };
  GroupRegs<NT, PRE> R[MAXB];
  // codes and scales of one batch of groups (load-time constants)
  auto load_weights = [&](int gb, int nb) {
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
        if (PRE && LAYOUT == 0) {
#pragma unroll
          for (int i = 0; i < 4; i++) R[u].ks[i] = load_ks(G * 128 + i * 32);
        }
      }
    }
  };
  // activations of one batch (written by the preceding kernel: only after the wait)
  auto load_acts = [&](int gb, int nb) {
    if (PRE) {
#pragma unroll
      for (int u = 0; u < MAXB; u++)
        if (u < nb)
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < NT; j++) R[u].xv[i][j] = load_x((gb + u) * 128 + i * 32, j);
    }
  };

  const bool early = a.const_weights != 0 && active_warp && gend > gbeg;
  if (early) {
    load_weights(gbeg, min(MAXB, gend - gbeg));  // overlaps the previous kernel's tail
  } else if (active_warp && t == 0 && gend > gbeg) {
    // weights may have been written by the previous kernel: only warm L2 before the wait
    if (oka) bulk_prefetch_l2(a.qs + (size_t)ra * RB + (size_t)gbeg * 64, (uint32_t)(gend - gbeg) * 64u);
    if (okb) bulk_prefetch_l2(a.qs + (size_t)rb * RB + (size_t)gbeg * 64, (uint32_t)(gend - gbeg) * 64u);
  }
  grid_dep_launch();
  grid_dep_wait();

  if (LN) {
    // LayerNorm statistics of this CTA's token rows, one warp per row: the
    // mean, then the mean of the centred squares (two passes, as the
    // reference's cpu_layernorm_stats, lold3344/ARIA src/transformer_cuda.rs:3276-3293)
    // (h is 16-byte aligned with ldx and K multiples of 4: float4 loads).
    // Rows of up to 1024 values are held in registers, so both passes cost
    // one round of loads; longer rows are read twice.
    const int nrow = min(8 * NT, a.M - m0);
    const int n4 = a.K >> 2;
    for (int tl = warp; tl < nrow; tl += 8) {
      const float4* hr = reinterpret_cast<const float4*>(a.h + (size_t)(m0 + tl) * a.ldx);
      float sum = 0.0f, sq = 0.0f, mean;
      if (n4 <= 8 * 32) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int c = lane + 32 * i;
          v[i] = c < n4 ? __ldg(hr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mean = sum / (float)a.K;
#pragma unroll
        for (int i = 0; i < 8; i++) {
          if (lane + 32 * i < n4) {
            const float c0 = v[i].x - mean, c1 = v[i].y - mean, c2 = v[i].z - mean, c3 = v[i].w - mean;
            sq = fmaf(c0, c0, sq);
            sq = fmaf(c1, c1, sq);
            sq = fmaf(c2, c2, sq);
            sq = fmaf(c3, c3, sq);
          }
        }
      } else {
        for (int c = lane; c < n4; c += 32) {
          const float4 v = __ldg(hr + c);
          sum += (v.x + v.y) + (v.z + v.w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mean = sum / (float)a.K;
        for (int c = lane; c < n4; c += 32) {
          const float4 v = __ldg(hr + c);
          const float c0 = v.x - mean, c1 = v.y - mean, c2 = v.z - mean, c3 = v.w - mean;
          sq = fmaf(c0, c0, sq);
          sq = fmaf(c1, c1, sq);
          sq = fmaf(c2, c2, sq);
          sq = fmaf(c3, c3, sq);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if (lane == 0) ln_stat[tl] = make_float2(mean, rsqrtf(sq / (float)a.K + a.ln_eps));
    }
    __syncthreads();
  }

  if (active_warp) {
    for (int gb = gbeg; gb < gend; gb += MAXB) {
      const int nb = min(MAXB, gend - gb);
      if (!(early && gb == gbeg)) load_weights(gb, nb);
      load_acts(gb, nb);
#pragma unroll
      for (int u = 0; u < MAXB; u++) {
        if (u >= nb) break;
        const int G = gb + u;
        const uint32_t qaw[4] = {R[u].qa.x, R[u].qa.y, R[u].qa.z, R[u].qa.w};
        const uint32_t qbw[4] = {R[u].qb.x, R[u].qb.y, R[u].qb.z, R[u].qb.w};
        uint4 ksg[4];
        if (!PRE && LAYOUT == 0) {
#pragma unroll
          for (int i = 0; i < 4; i++) ksg[i] = load_ks(G * 128 + i * 32);  // the group's KN scales at once
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int kb = G * 128 + i * 32;
          if (kb >= a.K) break;  // padded tail of K (uniform across the warp)
          uint4 xv[NT];
#pragma unroll
          for (int j = 0; j < NT; j++) xv[j] = PRE ? R[u].xv[PRE ? i : 0][PRE ? j : 0] : load_x(kb, j);
          if (LAYOUT == 0) {
            const uint4 s8 = PRE ? R[u].ks[PRE ? i : 0] : ksg[i];
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

  // Reduction over the K slices: the S warps of a tile in shared memory, then
  // (C > 1) the C CTAs of the cluster through distributed shared memory into
  // cluster rank 0.  Every thread reaches every barrier: no early return above.
  const bool leader = active_warp && ks == 0;
  if (S > 1 || C > 1) {
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) red[warp][lane][j * 4 + e] = acc[j][e];
    __syncthreads();
    if (leader) {
      for (int s2 = 1; s2 < S; s2++)
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
          for (int e = 0; e < 4; e++) acc[j][e] += red[warp + s2][lane][j * 4 + e];
    }
    if (C > 1) {
      __syncthreads();  // the leader rows of red are rewritten below
      if (leader) {
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
          for (int e = 0; e < 4; e++) red[warp][lane][j * 4 + e] = acc[j][e];
      }
      cluster_sync_all();  // every CTA's partial is in its shared memory
      if (leader && crank == 0) {
        for (int rr = 1; rr < C; rr++)
#pragma unroll
          for (int j = 0; j < NT; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[j][e] += ld_dsmem_f32(&red[warp][lane][j * 4 + e], (uint32_t)rr);
      }
      cluster_sync_all();  // peers keep their shared memory until rank 0 has read it
    }
  }
  if (!leader || crank != 0) return;

  // D fragment: c0,c1 -> (row g, tokens 2t, 2t+1); c2,c3 -> (row g+8, same tokens)
  float bia = 0.f, bib = 0.f;
  if (a.bias) {
    if (oka) bia = __half2float(a.bias[ra]);
    if (okb) bib = __half2float(a.bias[rb]);
  }
  float o[NT * 4];
#pragma unroll
  for (int j = 0; j < NT; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) o[4 * j + e] = a.alpha * acc[j][e] + (e >= 2 ? bib : bia);
  // element i = 4j + e: row ra (rb for e >= 2), token m0 + 8j + 2t + (e & 1)
  auto tok = [&](int i) { return m0 + 8 * (i >> 2) + 2 * t + (i & 1); };
  auto row = [&](int i) { return (i & 3) >= 2 ? rb : ra; };
  store_outputs<NT * 4>(
      a.y, a.ydt, o, a.beta,
      [&](int i) { return (size_t)min(tok(i), a.M - 1) * a.ldy + min(row(i), a.N - 1); },
      [&](int i) { return tok(i) < a.M && ((i & 3) >= 2 ? okb : oka); });
}

template <int LAYOUT, int NT, int MAXB, bool PRE, bool LN>
static cudaError_t launch_t2(const DecodeArgs& a, cudaStream_t st, bool pdl) {
  const int tiles = (a.N + 15) / 16;
  const int tpc = 8 / a.ksplit;
  dim3 grid(((tiles + tpc - 1) / tpc) * a.csplit, (a.M + 8 * NT - 1) / (8 * NT));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (a.csplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = a.csplit;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, decode_mma_kernel<LAYOUT, NT, MAXB, PRE, LN>, a);
}

template <int LAYOUT, int NT, int MAXB, bool PRE>
static cudaError_t launch_t(const DecodeArgs& a, cudaStream_t st, bool pdl) {
  if (a.h) return launch_t2<LAYOUT, NT, MAXB, PRE, true>(a, st, pdl);
  return launch_t2<LAYOUT, NT, MAXB, PRE, false>(a, st, pdl);
}

template <int LAYOUT>
static cudaError_t launch_layout(const DecodeArgs& a, int nt, int gpw, cudaStream_t st, bool pdl) {
  // register budget (128/thread at 2 CTAs per SM): preloading the activation
  // fragments is affordable for one or two token tiles
  if (nt == 1) return gpw <= 1 ? launch_t<LAYOUT, 1, 1, true>(a, st, pdl) : launch_t<LAYOUT, 1, 2, true>(a, st, pdl);
  if (nt == 2) return launch_t<LAYOUT, 2, 1, true>(a, st, pdl);
  if (nt == 4) return launch_t<LAYOUT, 4, 1, false>(a, st, pdl);
  return launch_t<LAYOUT, 8, 1, false>(a, st, pdl);
}

// Decode-regime projection for M <= 64 (larger M goes to the tcgen05 kernel).
// Work split: a 16-row tile's K is cut into `ksplit` slices (one warp each) when
// there are too few tiles to give every SM sixteen warps; if that still leaves
// SMs idle and K is long, a cluster of `csplit` CTAs splits K further and
// reduces through distributed shared memory.
cudaError_t launch_decode(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                          int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl,
                          bool const_weights, const float* ln_h, const __half* ln_g, const __half* ln_b,
                          float ln_eps) {
  DecodeArgs a;
  a.const_weights = const_weights ? 1 : 0;
  a.h = ln_h;
  a.ln_g = ln_g;
  a.ln_b = ln_b;
  a.ln_eps = ln_eps;
  a.qs = tiled;
  a.scales = reinterpret_cast<const __half*>(tiled + tiled_scale_offset(K, N));
  a.K = K; a.N = N; a.Kp = padded_k(K);
  a.x = x; a.ldx = ldx; a.M = M; a.y = y; a.ydt = ydt; a.ldy = ldy;
  a.bias = bias; a.alpha = alpha; a.beta = beta;
  const int KG = a.Kp / 128;
  const int tiles = (N + 15) / 16;
  int S = 1;
  while (S < 8 && S < KG && ((long long)tiles * S < 148LL * 16 || (KG + S - 1) / S > 2)) S++;
  int C = 1;
  const int ctas = (tiles + (8 / S) - 1) / (8 / S);
  while (C < 4 && (long long)ctas * C < 148 && KG >= 2 * S * C) C *= 2;
  a.ksplit = S;
  a.csplit = C;
  const int gpw = (KG + S * C - 1) / (S * C);
  // tokens per pass (8 NT): weights with few row tiles take 16-token passes at
  // any M (more warps in flight per SM; the weight stays in L2 between passes),
  // the others one pass of up to 64 (measured on B200 at M = 24..64: Efkolos
  // attn_out 2.6-2.8 us with NT = 2 against 3.6-9.0 with NT = 4 / 8, ffn_down
  // 5.5-10.3 against 7.6-15.9; QKV, ffn_up and the LM head the other way)
  const int nt = M <= 8 ? 1 : (M <= 16 || tiles <= kDecodeFewTiles) ? 2 : (M <= 32 ? 4 : 8);
  return layout == 1 ? launch_layout<1>(a, nt, gpw, st, pdl) : launch_layout<0>(a, nt, gpw, st, pdl);
}

}  // namespace aria_q4
