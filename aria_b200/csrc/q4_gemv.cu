// q4_gemv.cu -- streaming Q4_0 GEMV for the decode regime (M <= 8 token rows).
//
// Replaces, for Q4_0 weights and one decode step's handful of token rows, the
// cuBLAS fp16 GEMM that ARIA runs for every projection (`gemm()` at
// lold3344/ARIA src/transformer_cuda.rs:615-640; call sites :1583 QKV, :1686
// attn_out, :1753 ffn_up, :1805 ffn_down, :1864 LM head).  The product is bound
// by weight bytes (0.5625 B per weight), so the kernel is built around keeping
// enough of them in flight on every SM and dequantising them at that rate:
//
//  * Persistent grid: two CTAs (8 warps each) per SM when their shared memory
//    allows, else one; or clusters of C CTAs when the weight has few row tiles
//    and a tall K.  Cluster q owns row tiles q, q + clusters, ... (16*R output
//    features each); its C CTAs split K, and the 8 warps of a CTA split the
//    CTA's K range again.
//  * Every warp streams its own sequence of (row tile, 128-k group) chunks --
//    16*R rows x 64*P bytes of codes plus that chunk's scales -- through a
//    private ring of 6/(R*P) stages (2 when R*P = 4) with 16-byte cp.async
//    copies (55-74 KB of ring per CTA).  The ring runs across tile boundaries, so the stream
//    never drains until the CTA's last chunk.  No register is spent on bytes in
//    flight, and waiting is cp.async.wait_group on the warp's own copies: no
//    spin loop anywhere.
//  * The activations of the CTA's K range are staged once in shared memory.
//  * Maths as in the register-fed kernel: codes become exact (q-8) f16x2 values
//    with LOP3 + HSUB/HFMA, written straight into the A-fragment order of
//    m16n8k16 tensor-core MMAs (A = weights, B = activations, f32 accumulation).  NK scales: each 32-k block's MMA pair
//    starts from zero and is scaled in f32 (exact products, f32 sums).  KN scales
//    are folded into the activation fragment (x*s rounded to f16).
//  * Partial sums: after each row tile, every warp deposits its fragment in a
//    double-buffered shared array and one warp (tile index mod 8) reduces the 8
//    partials in a fixed order -- deterministic results.  With C > 1 the CTA
//    sums are kept per tile and added across the cluster through distributed
//    shared memory at the end.
//  * Programmatic dependent launch: when the caller declares the weights
//    constant, the first D chunks of every warp are requested before
//    griddepcontrol.wait, overlapping the previous kernel; otherwise the first
//    tile's rows are only prefetched to L2.
#include <algorithm>

#include "q4_common.cuh"

namespace aria_q4 {

struct GemvArgs {
  const uint8_t* qs;
  const __half* scales;
  int K, N, Kp, KG;
  const __half* x;
  int ldx, M;
  void* y;
  int ydt, ldy;
  const __half* bias;
  float alpha, beta;
  int tiles;      // row tiles of 16*R features
  int clusters;   // tile ranges (one per cluster, or per CTA when C == 1)
  int C;          // CTAs per cluster: K split
  int x_stride;   // halves per staged activation row
  int ring_slots; // ring stages per warp actually allocated (kDepth, or fewer when no warp has more chunks)
  int const_weights;
};

constexpr int kGemvWarps = 8;                     // warps of a CTA: they split each row tile's K range
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvMaxM = 8;
constexpr int kGemvMaxTilesCta = 16;              // tiles per cluster when C > 1 (cluster partial store)
constexpr size_t kGemvSmemMax = 227 * 1024;
constexpr size_t kGemvSmemHalf = 113 * 1024;     // two CTAs per SM: 228 KB less 1 KB reserved per CTA

// R: 16-row sub-tiles per row tile; P: 128-k groups per chunk (a chunk of P = 2
// reads whole 128-byte lines of every row and halves the per-chunk overhead).
template <int R, int P>
struct GemvShape {
  static constexpr int kWarps = kGemvWarps;
  static constexpr int kThreads = kGemvThreads;
  static constexpr int kDepth = R * P == 1 ? 6 : (R * P == 2 ? 3 : 2);  // stages per warp
  static constexpr int kCodeBytes = R * P * 1024;  // [P][16R rows][64 B]
  static constexpr int kStage = kCodeBytes + P * 256;  // + scales [P][NK: 16R rows x 8 B | KN: 128 k x 2 B]
  static constexpr int kRing = kWarps * kDepth * kStage;
  static constexpr int kRedFloats = 4 * R;         // per lane
  static constexpr int kRed = 2 * kGemvWarps * 32 * kRedFloats * 4;
  static constexpr int kRedCta = kGemvMaxTilesCta * 32 * kRedFloats * 4;
  // one-token partials of up to kGemvMaxTilesCta tiles (8 lanes x 2R floats per warp)
  static_assert(kGemvMaxTilesCta * kGemvWarps * 8 * 2 * R * 4 <= kRed, "deferred partials exceed the reduction area");
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ void bar_sync_warps(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ float4 ld_dsmem_v4(const float* local_addr, uint32_t rank) {
  uint32_t remote;
  float4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(tc_smem_u32(local_addr)), "r"(rank));
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}
// d = A*B with a zero accumulator (no register moves to clear it)
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                                            const uint32_t a3, const uint32_t b0, const uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// D fragment element e of a 16-row sub-tile: row g (+8 for e >= 2), token 2t + (e & 1)
template <int R>
__device__ __forceinline__ void gemv_store_tile(const GemvArgs& a, const float (&v)[R][4], const float (&bias)[R][2],
                                                int r0, int g, int t) {
  float o[4 * R];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int e = 0; e < 4; e++) o[4 * r + e] = a.alpha * v[r][e] + bias[r][e >> 1];
  // element i = 4r + e: row r0 + 16r + g (+8 for e >= 2), token 2t + (e & 1)
  auto row = [&](int i) { return r0 + 16 * (i >> 2) + g + ((i & 3) >= 2 ? 8 : 0); };
  auto tok = [&](int i) { return 2 * t + (i & 1); };
  store_outputs<4 * R>(
      a.y, a.ydt, o, a.beta,
      [&](int i) { return (size_t)min(tok(i), a.M - 1) * a.ldy + min(row(i), a.N - 1); },
      [&](int i) { return tok(i) < a.M && row(i) < a.N; });
}


template <int R>
__device__ __forceinline__ void gemv_load_bias(const GemvArgs& a, float (&b)[R][2], int r0, int g) {
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int n = r0 + 16 * r + g + 8 * h;
      b[r][h] = (a.bias && n < a.N) ? __half2float(a.bias[n]) : 0.0f;
    }
}

// ONE: a single token row (M = 1), NK only: the block-scale FMAs of the unused
// odd token columns are left out.
template <int LAYOUT, int R, int P, bool ONE = false>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_stream_kernel(const GemvArgs a) {
  using S = GemvShape<R, P>;
  constexpr int D = S::kDepth;
  constexpr int TR = 16 * R;  // rows per tile
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t ring_base = tc_smem_u32(smem);
  const uint32_t ring_bytes = (uint32_t)(S::kWarps * a.ring_slots * S::kStage);
  float* red = reinterpret_cast<float*>(smem + ring_bytes);
  float* red_cta = reinterpret_cast<float*>(smem + ring_bytes + S::kRed);
  const uint32_t xs_base = tc_smem_u32(smem + ring_bytes + S::kRed + (a.C > 1 ? S::kRedCta : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int C = a.C;
  const int crank = (int)blockIdx.x % C;
  const int q = (int)blockIdx.x / C;
  // row tiles q, q + clusters, q + 2 clusters, ...: at any moment the clusters
  // stream neighbouring tiles, so the weight reads advance through memory as one front
  const int tstep = a.clusters;
  const int ntl = q < a.tiles ? (a.tiles - 1 - q) / tstep + 1 : 0;
  const int gc0 = crank * a.KG / C, gc1 = (crank + 1) * a.KG / C;
  const int gw0 = gc0 + warp * (gc1 - gc0) / kGemvWarps;
  const int gw1 = gc0 + (warp + 1) * (gc1 - gc0) / kGemvWarps;
  const int ns = (gw1 - gw0 + P - 1) / P;  // chunks per tile; the last one may hold fewer than P groups
  const size_t RB = (size_t)a.Kp >> 1;
  // a warp never has more chunks than ring_slots when ring_slots < D, so its
  // stage index (counted modulo D) stays below ring_slots
  const uint32_t my_ring = ring_base + (uint32_t)(warp * a.ring_slots) * S::kStage;

  // Issue side of the warp's ring: chunk (tile is_j, groups is_G .. is_G+P-1)
  // goes to stage is_slot.  Code piece c = lane + 32u (16 bytes) is row
  // c / (4P), group (c / 4) % P, column c % 4, so each copy instruction reads
  // whole 64P-byte row segments (8/P rows per instruction).  Source pointers
  // advance incrementally; chunks inside N and inside the warp's slice (all but
  // the edges) take an unpredicated path.
  constexpr int kRowsPerCopy = 8 / P;
  constexpr int kScalePieces = LAYOUT == 1 ? (P * TR + 31) / 32 : 1;
  const int lane_row = lane / (4 * P), lane_grp = (lane >> 2) % P, lane_col = lane & 3;
  const uint8_t* lane_qs = a.qs + (size_t)lane_row * RB + lane_grp * 64 + lane_col * 16;
  const uint32_t lane_dst = (uint32_t)(lane_grp * TR * 64 + lane_row * 64 + lane_col * 16);
  const size_t copy_step = (size_t)kRowsPerCopy * RB;
  // scale pieces of this lane: NK -> (group h, row) pairs of 8 bytes; KN -> 16 bytes (lanes < 16P)
  int sc_row[kScalePieces], sc_h[kScalePieces];
  size_t sc_off[kScalePieces];
#pragma unroll
  for (int v = 0; v < kScalePieces; v++) {
    const int pc = lane + 32 * v;
    sc_h[v] = LAYOUT == 1 ? pc / TR : lane >> 4;
    sc_row[v] = LAYOUT == 1 ? pc % TR : 0;
    sc_off[v] = LAYOUT == 1 ? ((size_t)sc_h[v] * a.N + sc_row[v]) * 4 : (size_t)lane * 8;
  }
  const bool sc_lane = LAYOUT == 1 ? lane < P * TR : lane < 16 * P;  // lane has a first scale piece
  int is_j = q, is_s = 0, is_slot = 0, is_G = gw0;
  const uint8_t* is_src = lane_qs + (size_t)is_j * TR * RB + (size_t)gw0 * 64;
  const __half* is_ssrc = LAYOUT == 1 ? a.scales + ((size_t)gw0 * a.N + (size_t)is_j * TR) * 4
                                      : a.scales + (size_t)((is_j * TR) >> 5) * a.Kp + (size_t)gw0 * 128;
  auto issue_next = [&]() {
    if (is_j < a.tiles && ns > 0) {
      const int r0 = is_j * TR;
      const uint32_t st = my_ring + (uint32_t)is_slot * S::kStage + lane_dst;
      const uint32_t sst = my_ring + (uint32_t)is_slot * S::kStage + S::kCodeBytes;
      const bool full_grp = P == 1 || is_G + P <= gw1;
      if (full_grp && r0 + TR <= a.N) {
        const uint8_t* src = is_src;
#pragma unroll
        for (int u = 0; u < 2 * R * P; u++) {
          cp_async16(st + (uint32_t)(kRowsPerCopy * u * 64), src, 16u);
          src += copy_step;
        }
        if (LAYOUT == 1) {
#pragma unroll
          for (int v = 0; v < kScalePieces; v++)
            if (v > 0 || sc_lane) cp_async8(sst + (uint32_t)(sc_h[v] * TR + sc_row[v]) * 8, is_ssrc + sc_off[v], 8u);
        } else if (sc_lane) {
          cp_async16(sst + (uint32_t)lane * 16, is_ssrc + sc_off[0], 16u);
        }
      } else {
        const bool grp_ok = P == 1 || is_G + lane_grp < gw1;
        const uint8_t* src = is_src;
#pragma unroll
        for (int u = 0; u < 2 * R * P; u++) {
          const bool ok = grp_ok && r0 + lane_row + kRowsPerCopy * u < a.N;
          cp_async16(st + (uint32_t)(kRowsPerCopy * u * 64), ok ? src : a.qs, ok ? 16u : 0u);
          src += copy_step;
        }
        if (LAYOUT == 1) {
#pragma unroll
          for (int v = 0; v < kScalePieces; v++)
            if (v > 0 || sc_lane) {
              const bool ok = r0 + sc_row[v] < a.N && is_G + sc_h[v] < gw1;
              cp_async8(sst + (uint32_t)(sc_h[v] * TR + sc_row[v]) * 8, ok ? is_ssrc + sc_off[v] : a.scales,
                        ok ? 8u : 0u);
            }
        } else if (sc_lane) {
          const bool ok = is_G + sc_h[0] < gw1;
          cp_async16(sst + (uint32_t)lane * 16, ok ? is_ssrc + sc_off[0] : a.scales, ok ? 16u : 0u);
        }
      }
      // advance to the next chunk of the warp's sequence
      if (++is_s == ns) {
        is_s = 0;
        is_j += tstep;
        is_G = gw0;
        is_src = lane_qs + (size_t)is_j * TR * RB + (size_t)gw0 * 64;
        is_ssrc = LAYOUT == 1 ? a.scales + ((size_t)gw0 * a.N + (size_t)is_j * TR) * 4
                              : a.scales + (size_t)((is_j * TR) >> 5) * a.Kp + (size_t)gw0 * 128;
      } else {
        is_G += P;
        is_src += 64 * P;
        is_ssrc += LAYOUT == 1 ? (size_t)P * a.N * 4 : (size_t)P * 128;
      }
      if (++is_slot == D) is_slot = 0;
    }
    cp_async_commit();
  };

  if (a.const_weights) {
#pragma unroll
    for (int i = 0; i < D; i++) issue_next();
  } else if (ns > 0 && ntl > 0 && lane < TR) {
    // warm L2 with this warp's slice of the first tile (rows may be written by the previous kernel)
    const int n = q * TR + lane;
    if (n < a.N) bulk_prefetch_l2(a.qs + (size_t)n * RB + (size_t)gw0 * 64, (uint32_t)(gw1 - gw0) * 64u);
  }
  grid_dep_launch();
  grid_dep_wait();

  // activations of the CTA's K range: rows 0..M-1, zero past K
  {
    const int kc0 = gc0 * 128;
    const int per_row = (gc1 - gc0) * 16;  // 16-byte pieces per row
    for (int c = threadIdx.x; c < a.M * per_row; c += kGemvThreads) {
      const int m = c / per_row, p = c - m * per_row;
      const int k = kc0 + p * 8;
      const bool ok = k < a.K;
      cp_async16(xs_base + (uint32_t)(m * a.x_stride + p * 8) * 2, ok ? a.x + (size_t)m * a.ldx + k : a.x,
                 ok ? 16u : 0u);
    }
    cp_async_commit();
  }
  if (!a.const_weights) {
#pragma unroll
    for (int i = 0; i < D; i++) issue_next();
  }
  // bias of the first tile this warp stores (tile number warp), loaded while the copies fly
  const int pre_tile = warp;
  float bias_pre[R][2];
  gemv_load_bias<R>(a, bias_pre, (q + pre_tile * tstep) * TR, g);
  cp_async_wait<0>();
  __syncthreads();

  // One token row and one CTA per tile range: no barrier per tile.  Each
  // warp's partial sums of every tile are kept (2R floats for each of the 8
  // lanes of token column 0, at most 16 tiles: within the double-buffered
  // reduction area) and reduced after the last tile, in the same fixed order.
  const bool defer = a.M == 1 && C == 1 && ntl <= kGemvMaxTilesCta;
  // lanes of token columns >= M read row 0: their MMA columns are never stored
  const uint32_t xrow = xs_base + (uint32_t)((g < a.M ? g : 0) * a.x_stride) * 2 + (uint32_t)(16 * t);
  int cs_slot = 0;
  for (int jl = 0; jl < ntl; jl++) {
    float acc[R][4];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int e = 0; e < 4; e++) acc[r][e] = 0.0f;

    for (int s = 0; s < ns; s++) {
      cp_async_wait<D - 1>();
      __syncwarp();
      const int G0 = gw0 + P * s;
      const uint32_t st = my_ring + (uint32_t)cs_slot * S::kStage;
      if (++cs_slot == D) cs_slot = 0;
#pragma unroll
      for (int h = 0; h < P; h++) {
        // Groups past K hold codes 8 (value 0) and zero activations: no tail test
        // is needed inside a group.  A chunk's missing last group is skipped.
        if (P > 1 && h > 0 && G0 + h >= gw1) break;
        const uint32_t sth = st + (uint32_t)(h * TR * 64);
        uint4 qa[R], qb[R];
        float sa[R][4], sb[R][4];
#pragma unroll
        for (int r = 0; r < R; r++) {
          qa[r] = lds128(sth + (uint32_t)((16 * r + g) * 64 + 16 * t));
          qb[r] = lds128(sth + (uint32_t)((16 * r + 8 + g) * 64 + 16 * t));
          if (LAYOUT == 1) {
            const uint32_t sc = st + S::kCodeBytes + (uint32_t)(h * TR) * 8;
            const uint2 wa = lds64(sc + (16 * r + g) * 8);
            const uint2 wb = lds64(sc + (16 * r + 8 + g) * 8);
            const float2 a01 = __half22float2(*reinterpret_cast<const __half2*>(&wa.x));
            const float2 a23 = __half22float2(*reinterpret_cast<const __half2*>(&wa.y));
            const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&wb.x));
            const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&wb.y));
            sa[r][0] = a01.x; sa[r][1] = a01.y; sa[r][2] = a23.x; sa[r][3] = a23.y;
            sb[r][0] = b01.x; sb[r][1] = b01.y; sb[r][2] = b23.x; sb[r][3] = b23.y;
          }
        }
        const uint32_t xg = xrow + (uint32_t)((G0 + h - gc0) * 256);
#pragma unroll
        for (int i4 = 0; i4 < 4; i4++) {
          uint4 xv = lds128(xg + i4 * 64);
          if (LAYOUT == 0) {
            const uint4 s8 = lds128(st + S::kCodeBytes + (uint32_t)(h * 256 + (32 * i4 + 8 * t) * 2));
            xv.x = hmul2_u32(xv.x, s8.x);
            xv.y = hmul2_u32(xv.y, s8.y);
            xv.z = hmul2_u32(xv.z, s8.z);
            xv.w = hmul2_u32(xv.w, s8.w);
          }
#pragma unroll
          for (int r = 0; r < R; r++) {
            const uint32_t wa = i4 == 0 ? qa[r].x : (i4 == 1 ? qa[r].y : (i4 == 2 ? qa[r].z : qa[r].w));
            const uint32_t wb = i4 == 0 ? qb[r].x : (i4 == 1 ? qb[r].y : (i4 == 2 ? qb[r].z : qb[r].w));
            uint32_t A1[4], A2[4];
            dequant_pair_mma(wa, wb, A1, A2);
            if (LAYOUT == 1) {
              float c[4];
              mma_16816_z(c, A1[0], A1[1], A1[2], A1[3], xv.x, xv.y);
              mma_16816(c, A2[0], A2[1], A2[2], A2[3], xv.z, xv.w);
              // c[1], c[3] are token column 2t + 1 >= 1: not needed for one token
              acc[r][0] = fmaf(sa[r][i4], c[0], acc[r][0]);
              acc[r][2] = fmaf(sb[r][i4], c[2], acc[r][2]);
              if (!ONE) {
                acc[r][1] = fmaf(sa[r][i4], c[1], acc[r][1]);
                acc[r][3] = fmaf(sb[r][i4], c[3], acc[r][3]);
              }
            } else {
              mma_16816(acc[r], A1[0], A1[1], A1[2], A1[3], xv.x, xv.y);
              mma_16816(acc[r], A2[0], A2[1], A2[2], A2[3], xv.z, xv.w);
            }
          }
        }
      }
      __syncwarp();  // every lane has read the stage before it is refilled
      issue_next();
    }

    if (defer) {
      // one token: only lanes of token column 0 (t == 0) hold outputs; their
      // partials wait in shared memory until every tile of the CTA is done
      if (t == 0) {
        float* mine = red + ((jl * kGemvWarps + warp) * 8 + g) * (2 * R);
#pragma unroll
        for (int r = 0; r < R; r++) {
          mine[2 * r] = acc[r][0];
          mine[2 * r + 1] = acc[r][2];
        }
      }
      continue;
    }
    // deposit this warp's partial, reduce the 8 warps' partials in a fixed order
    float* mine = red + (((jl & 1) * kGemvWarps + warp) * 32 + lane) * S::kRedFloats;
#pragma unroll
    for (int r = 0; r < R; r++)
      *reinterpret_cast<float4*>(mine + 4 * r) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    bar_sync_warps(1, kGemvThreads);
    if (warp == (jl & (kGemvWarps - 1))) {
      float tot[R][4];
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int e = 0; e < 4; e++) tot[r][e] = 0.0f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; w++) {
        const float* pp = red + (((jl & 1) * kGemvWarps + w) * 32 + lane) * S::kRedFloats;
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float4 v = *reinterpret_cast<const float4*>(pp + 4 * r);
          tot[r][0] += v.x; tot[r][1] += v.y; tot[r][2] += v.z; tot[r][3] += v.w;
        }
      }
      if (C > 1) {
        float* dst = red_cta + (jl * 32 + lane) * S::kRedFloats;
#pragma unroll
        for (int r = 0; r < R; r++)
          *reinterpret_cast<float4*>(dst + 4 * r) = make_float4(tot[r][0], tot[r][1], tot[r][2], tot[r][3]);
      } else {
        float bia[R][2];
        if (jl == pre_tile) {
#pragma unroll
          for (int r = 0; r < R; r++) { bia[r][0] = bias_pre[r][0]; bia[r][1] = bias_pre[r][1]; }
        } else {
          gemv_load_bias<R>(a, bia, (q + jl * tstep) * TR, g);
        }
        gemv_store_tile<R>(a, tot, bia, (q + jl * tstep) * TR, g, t);
      }
    }
  }

  if (defer) {
    bar_sync_warps(1, kGemvThreads);
    for (int jl = warp; jl < ntl; jl += kGemvWarps) {
      float tot[R][4];
#pragma unroll
      for (int r = 0; r < R; r++)
#pragma unroll
        for (int e = 0; e < 4; e++) tot[r][e] = 0.0f;
      if (t == 0) {
#pragma unroll
        for (int w = 0; w < kGemvWarps; w++) {
          const float* pp = red + ((jl * kGemvWarps + w) * 8 + g) * (2 * R);
#pragma unroll
          for (int r = 0; r < R; r++) {
            tot[r][0] += pp[2 * r];
            tot[r][2] += pp[2 * r + 1];
          }
        }
      }
      float bia[R][2];
      if (jl == pre_tile) {
#pragma unroll
        for (int r = 0; r < R; r++) { bia[r][0] = bias_pre[r][0]; bia[r][1] = bias_pre[r][1]; }
      } else {
        gemv_load_bias<R>(a, bia, (q + jl * tstep) * TR, g);
      }
      gemv_store_tile<R>(a, tot, bia, (q + jl * tstep) * TR, g, t);
    }
  }

  if (C > 1) {
    // every CTA's per-tile sums are in its shared memory: cluster rank 0 adds them
    // in rank order (all peers' loads issued before the first add)
    cluster_sync_all();
    if (crank == 0) {
      for (int jl = warp; jl < ntl; jl += kGemvWarps) {
        const float* pp = red_cta + (jl * 32 + lane) * S::kRedFloats;
        float4 pv[3][R];
#pragma unroll
        for (int rr = 1; rr < 4; rr++)
          if (rr < C)
#pragma unroll
            for (int r = 0; r < R; r++) pv[rr - 1][r] = ld_dsmem_v4(pp + 4 * r, (uint32_t)rr);
        float tot[R][4];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const float4 v = *reinterpret_cast<const float4*>(pp + 4 * r);
          tot[r][0] = v.x; tot[r][1] = v.y; tot[r][2] = v.z; tot[r][3] = v.w;
        }
#pragma unroll
        for (int rr = 1; rr < 4; rr++)
          if (rr < C)
#pragma unroll
            for (int r = 0; r < R; r++) {
              tot[r][0] += pv[rr - 1][r].x; tot[r][1] += pv[rr - 1][r].y;
              tot[r][2] += pv[rr - 1][r].z; tot[r][3] += pv[rr - 1][r].w;
            }
        float bia[R][2];
        if (jl == pre_tile) {
#pragma unroll
          for (int r = 0; r < R; r++) { bia[r][0] = bias_pre[r][0]; bia[r][1] = bias_pre[r][1]; }
        } else {
          gemv_load_bias<R>(a, bia, (q + jl * tstep) * TR, g);
        }
        gemv_store_tile<R>(a, tot, bia, (q + jl * tstep) * TR, g, t);
      }
    }
    cluster_sync_all();  // peers keep their shared memory until rank 0 has read it
  }
}

// ------------------------------------------------------------------ launch

// ring stages per warp: the full depth, or the longest warp's chunk count when smaller
template <int R, int P>
static int gemv_ring_slots(long long chunks_per_warp) {
  return (int)std::min<long long>(GemvShape<R, P>::kDepth, std::max<long long>(1, chunks_per_warp));
}

template <int R, int P>
static size_t gemv_smem(int C, size_t xbytes, long long chunks_per_warp) {
  using S = GemvShape<R, P>;
  return (size_t)S::kWarps * gemv_ring_slots<R, P>(chunks_per_warp) * S::kStage + S::kRed +
         (C > 1 ? S::kRedCta : 0) + xbytes;
}

static int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
  return sms;
}

struct GemvPlan {
  int R = 0, P = 1, C = 1, tiles = 0, clusters = 0, x_stride = 0, ring_slots = 1;
  size_t smem = 0;
};

// One-time (per device) attributes of a kernel instance: all of shared memory
// may be requested, and the carveout keeps the SM in one configuration across a
// chain of projections, so the next kernel's CTA can become resident beside this one.
template <int LAYOUT, int R, int P, bool ONE = false>
static cudaError_t gemv_configure() {
  static int configured_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (configured_dev == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(gemv_stream_kernel<LAYOUT, R, P, ONE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kGemvSmemMax);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemv_stream_kernel<LAYOUT, R, P, ONE>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  configured_dev = dev;
  return cudaSuccess;
}

// Clusters of C CTAs that can be resident at once with per_sm CTAs' worth of
// shared memory each.  A cluster must fit inside one GPC, so on a part whose
// GPCs hold unequal SM counts fewer than sms * per_sm / C fit (B200: 33 clusters
// of 4 at one CTA per SM, 71 at two, but all 74 / 148 clusters of 2); a plan
// beyond this count would run a second wave.  Cached per device.
template <int LAYOUT, int R, int P>
static int gemv_max_clusters_t(int C, int per_sm, int fallback) {
  if (gemv_configure<LAYOUT, R, P>() != cudaSuccess) {
    cudaGetLastError();
    return fallback;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C * 64);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = per_sm == 2 ? kGemvSmemHalf : kGemvSmemMax;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemv_stream_kernel<LAYOUT, R, P>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return fallback;
  }
  return n;
}

static int gemv_max_clusters(int layout, int R, int P, int C, int per_sm, int sms) {
  const int fallback = std::max(1, sms * per_sm / C);
  if (C == 1) return fallback;
  constexpr int kDevices = 64;
  static int cache[kDevices][2][2][2][2][2];  // [dev][layout][R-1][P-1][C==4][per_sm-1]; 0 = not queried
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevices) {
    cudaGetLastError();
    return fallback;
  }
  int& slot = cache[dev][layout & 1][R - 1][P - 1][C == 4 ? 1 : 0][per_sm - 1];
  if (slot == 0) {
    // not a stream operation; relaxed capture mode keeps a first call made while
    // the thread captures a CUDA graph from invalidating that capture
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    int n;
    if (layout == 1)
      n = R == 2 ? (P == 2 ? gemv_max_clusters_t<1, 2, 2>(C, per_sm, fallback) : gemv_max_clusters_t<1, 2, 1>(C, per_sm, fallback))
                 : (P == 2 ? gemv_max_clusters_t<1, 1, 2>(C, per_sm, fallback) : gemv_max_clusters_t<1, 1, 1>(C, per_sm, fallback));
    else
      n = R == 2 ? (P == 2 ? gemv_max_clusters_t<0, 2, 2>(C, per_sm, fallback) : gemv_max_clusters_t<0, 2, 1>(C, per_sm, fallback))
                 : (P == 2 ? gemv_max_clusters_t<0, 1, 2>(C, per_sm, fallback) : gemv_max_clusters_t<0, 1, 1>(C, per_sm, fallback));
    cudaThreadExchangeStreamCaptureMode(&mode);
    slot = std::min(n, fallback);
  }
  return slot;
}

// Picks the tile height (16 or 32 rows), the groups per chunk (1 or 2), the
// cluster K split (1, 2 or 4) and two or one CTAs per SM (two when their
// shared memory allows).  Cost model, fitted to timings of every feasible plan
// of the Efkolos and d_model-4096 projections at M = 1 and 8 on B200 (chains of
// launches, weights larger than L2; the chosen plan is within 2% of the fastest
// on average, 8.5% at worst), in units of ~3.5 ns:
//   chunks of the longest warp x (100 + 150 per 16-row x 128-k block)
//     (x1.4 when two CTAs share an SM)
//   + 300 per row tile of a CTA (partial-sum reduction and store)
//   + 20 per token row and 128-k group of activations staged per SM (the
//     prologue copies them from L2 before the weight stream starts); 8 for a
//     single row (refit at M = 1 after the per-tile barrier was removed: the
//     chosen plan is within 0.3% of the fastest of every feasible plan on the
//     Efkolos ffn_down / LM head and config-4 attn_out / ffn_down / QKV / LM
//     head, against 2% with 20 -- config-4 attn_out 4.76 -> 4.33 us)
//   + 3000 for a cluster split (cluster barriers, distributed-shared-memory sums).
// Time is set by each warp's chain of chunk arrival -> dequantisation -> MMA ->
// scale FMAs (without the arithmetic the same copies stream ~1.8x faster), so the
// terms count a warp's chunks and blocks rather than bytes.
static bool plan_gemv(int layout, int K, int N, int M, int sms, GemvPlan& best) {
  const int KG = padded_k(K) / 128;
  long long best_cost = -1;
  for (int C : {1, 2, 4}) {
    if (C > KG) continue;
    const int gmax = (KG + C - 1) / C;
    const int gw = (gmax + kGemvWarps - 1) / kGemvWarps;  // groups of the longest warp slice
    const int x_stride = gmax * 128 + 8;  // 16-byte row pad: rows start in different banks
    const size_t xbytes = (size_t)M * x_stride * 2;
    for (int R : {2, 1}) {
      for (int P : {2, 1}) {
        if (P == 2 && gw < 2) continue;
        const int tiles = (N + 16 * R - 1) / (16 * R);
        for (int per_sm : {2, 1}) {
          const int clusters = std::min(tiles, gemv_max_clusters(layout, R, P, C, per_sm, sms));
          const int tpc = (tiles + clusters - 1) / clusters;
          if (C > 1 && tpc > kGemvMaxTilesCta) continue;
          const long long chunks = (long long)tpc * ((gw + P - 1) / P);  // per warp
          const size_t smem = R == 2 ? (P == 2 ? gemv_smem<2, 2>(C, xbytes, chunks) : gemv_smem<2, 1>(C, xbytes, chunks))
                                     : (P == 2 ? gemv_smem<1, 2>(C, xbytes, chunks) : gemv_smem<1, 1>(C, xbytes, chunks));
          if (smem > (per_sm == 2 ? kGemvSmemHalf : kGemvSmemMax)) continue;
          const int ctas_per_sm = std::min(per_sm, (clusters * C + sms - 1) / sms);
          const long long x_cost = M == 1 ? 8 : 20;
          const long long cost = chunks * (100 + 150 * R * P) * (per_sm == 2 ? 7 : 5) / 5 + 300LL * tpc +
                                 x_cost * ctas_per_sm * M * gmax + (C > 1 ? 3000 : 0);
          if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best.R = R;
            best.P = P;
            best.C = C;
            best.tiles = tiles;
            best.clusters = clusters;
            best.x_stride = x_stride;
            best.ring_slots = R == 2 ? (P == 2 ? gemv_ring_slots<2, 2>(chunks) : gemv_ring_slots<2, 1>(chunks))
                                     : (P == 2 ? gemv_ring_slots<1, 2>(chunks) : gemv_ring_slots<1, 1>(chunks));
            best.smem = smem;
          }
        }
      }
    }
  }
  return best_cost >= 0;
}

template <int LAYOUT, int R, int P, bool ONE>
static cudaError_t launch_gemv_t(const GemvArgs& a, size_t smem, cudaStream_t st, bool pdl) {
  cudaError_t e = gemv_configure<LAYOUT, R, P, ONE>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.clusters * a.C);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (a.C > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = a.C;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<LAYOUT, R, P, ONE>, a);
}

template <int LAYOUT>
static cudaError_t launch_gemv_layout(const GemvArgs& a, const GemvPlan& p, cudaStream_t st, bool pdl) {
  constexpr bool kNK = LAYOUT == 1;
  if (kNK && a.M == 1) {
    if (p.R == 2) return p.P == 2 ? launch_gemv_t<LAYOUT, 2, 2, kNK>(a, p.smem, st, pdl)
                                  : launch_gemv_t<LAYOUT, 2, 1, kNK>(a, p.smem, st, pdl);
    return p.P == 2 ? launch_gemv_t<LAYOUT, 1, 2, kNK>(a, p.smem, st, pdl)
                    : launch_gemv_t<LAYOUT, 1, 1, kNK>(a, p.smem, st, pdl);
  }
  if (p.R == 2) return p.P == 2 ? launch_gemv_t<LAYOUT, 2, 2, false>(a, p.smem, st, pdl)
                                : launch_gemv_t<LAYOUT, 2, 1, false>(a, p.smem, st, pdl);
  return p.P == 2 ? launch_gemv_t<LAYOUT, 1, 2, false>(a, p.smem, st, pdl)
                  : launch_gemv_t<LAYOUT, 1, 1, false>(a, p.smem, st, pdl);
}

// true when the streaming kernel takes this shape (M <= 8 and the CTA's
// activation slice fits in shared memory)
bool gemv_supported(int K, int N, int M) {
  if (M < 1 || M > kGemvMaxM) return false;
  GemvPlan p;
  return plan_gemv(0, K, N, M, device_sms(), p) && plan_gemv(1, K, N, M, device_sms(), p);
}

cudaError_t launch_gemv(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                        int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl,
                        bool const_weights) {
  GemvPlan p;
  if (!plan_gemv(layout, K, N, M, device_sms(), p)) return cudaErrorInvalidValue;
  GemvArgs a;
  a.qs = tiled;
  a.scales = reinterpret_cast<const __half*>(tiled + tiled_scale_offset(K, N));
  a.K = K; a.N = N; a.Kp = padded_k(K); a.KG = a.Kp / 128;
  a.x = x; a.ldx = ldx; a.M = M;
  a.y = y; a.ydt = ydt; a.ldy = ldy;
  a.bias = bias; a.alpha = alpha; a.beta = beta;
  a.tiles = p.tiles; a.clusters = p.clusters; a.C = p.C; a.x_stride = p.x_stride; a.ring_slots = p.ring_slots;
  a.const_weights = const_weights ? 1 : 0;
  return layout == 1 ? launch_gemv_layout<1>(a, p, st, pdl) : launch_gemv_layout<0>(a, p, st, pdl);
}

}  // namespace aria_q4
