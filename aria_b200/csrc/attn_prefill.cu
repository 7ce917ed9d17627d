// attn_prefill.cu -- causal attention over whole prompts on the 5th-generation
// tensor cores (tcgen05, sm_100a).
//
// The reference's forward pass recomputes attention over the whole prompt every
// step; its flash-attention forward (lold3344/ARIA src/kernels.cu:1298-1437,
// `flash_attn_fwd`: q, k, v, out [NH][T][dh] f16, lse [NH][T], causal, online
// softmax, one thread per head dimension) is SIMT.  This kernel computes the
// same outputs -- out = softmax(scale q k^T, causal) v and lse = max + ln(sum)
// per query row -- with the products on the tensor cores:
//
// Persistent: one CTA per SM walks the (sequence, head, 128-query tile) work
// items, heaviest tiles first, round-robin.  For every 128-key block j of a
// tile, up to the diagonal:
//   S_j = Q K_j^T     tcgen05.mma, A = Q tile and B = K block from shared memory
//                     (TMA, 128-byte swizzle), f32 S in tensor memory (128 x 128)
//   P_j = exp2(S_j - m) per row, written as f16 over S_j's own TMEM columns
//   O_j = P_j V_j     tcgen05.mma, A = P from tensor memory, B = V_j^T from
//                     shared memory (K-major: keys contiguous), into a fresh
//                     TMEM accumulator (128 x dh)
// and the running output O = O alpha_j + O_j (alpha_j = exp2(m_{j-1} - m_j))
// is kept in registers, so no accumulator in tensor memory ever needs
// rescaling.  Twelve warps, specialised (at most 3 per SM sub-partition, so
// each thread may hold up to 168 registers: the output row lives in them):
//   warp 0      TMA producer: the Q tile once, K blocks into a 2-stage ring, V
//               blocks into one buffer (freed by the transposers)
//   warp 1      TMEM allocator + single-thread MMA issuer (S_{j+1} is issued
//               before O_j, so the softmax of one block overlaps the product of
//               the previous one)
//   warps 2-9   softmax and output: two warps per TMEM lane quadrant, one per
//               half of the 128 keys (row max exchanged through shared memory)
//               and of the dh output columns; thread = query row
//   warps 10-11 V transposers: 8x8 blocks through ldmatrix.trans / stmatrix into
//               the K-major V^T operand
// The Q tile and the K/V blocks are TMA boxes of a 4-D view {dh, head, position,
// sequence}, so one kernel reads both the reference's [NH][T][dh] tensors and
// the packed [tokens][3 d] output of the QKV projection; positions past T read
// as zeros.  Every wait is bounded (the projection kernel's scheme: one second
// for the MMA issuer, two for the others, an abort flag, the error code in this
// unit's g_device_error).
#include <cuda.h>

#include <cstring>

#include "q4_common.cuh"
#include "q4_tcgen05.cuh"

namespace aria_q4 {

constexpr int kAttnThreads = 384;
constexpr int kBQ = 128;  // query rows per CTA (TMEM lanes)
constexpr int kBK = 128;  // keys per block

struct AttnArgs {
  int T, H, B;   // positions per sequence, heads, sequences
  float scale_log2;  // scale * log2(e)
  __half* out;
  long long o_seq, o_head, o_pos;  // element strides of out
  float* lse;                      // optional [B][H][T] (natural log)
  int n_qt;                        // query tiles per sequence
  unsigned long long wait_ns;
  int fill_cache;                  // store every K and V block into the caches (tm_kc, tm_vc)
};

template <int DH>
struct AttnSmem {
  static constexpr int kQ = kBQ * DH * 2;    // Q tile: DH / 64 boxes of [128 rows][128 B]
  static constexpr int kKV = kBK * DH * 2;   // one K (or V, or V^T) block
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQ;               // [2] K stages
  static constexpr int kVOff = kKOff + 2 * kKV;          // V block (one: the transposers turn it over fast)
  static constexpr int kVtOff = kVOff + kKV;             // [2] V^T stages: 2 boxes of [DH rows][128 B]
  static constexpr int kRedOff = kVtOff + 2 * kKV;       // row-max exchange [2 parity][2 halves][128] f32
  static constexpr int kSumOff = kRedOff + 2 * 2 * kBQ * 4;  // row-sum exchange [2 halves][128] f32
  static constexpr int kBarOff = kSumOff + 2 * kBQ * 4;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

// Query tile t of the persistent schedule: heaviest (last) tiles first.
struct AttnTile {
  int seq, head, q0, nb;
};
__device__ __forceinline__ AttnTile attn_tile(const AttnArgs& a, int t) {
  const int bh_count = a.B * a.H;
  const int qt = a.n_qt - 1 - t / bh_count;
  const int bh = t % bh_count;
  AttnTile r;
  r.seq = bh / a.H;
  r.head = bh % a.H;
  r.q0 = qt * kBQ;
  r.nb = min(qt + 1, (a.T + kBK - 1) / kBK);  // key blocks up to the diagonal
  return r;
}

template <int DH>
__global__ void __maxnreg__(168)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kc,
                        const __grid_constant__ CUtensorMap tm_vc, const AttnArgs a) {
  using L = AttnSmem<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_empty = q_full + 1;    // S MMA commit after a tile's last block
  uint64_t* k_full = q_empty + 1;    // [2]
  uint64_t* k_empty = k_full + 2;    // [2] S MMA commit (+ transposer warp 0 when filling the caches)
  uint64_t* v_full = k_empty + 2;    // [1]
  uint64_t* v_empty = v_full + 1;    // [1] 2 transposer warps
  uint64_t* vt_full = v_empty + 1;   // [2] 2 transposer warps
  uint64_t* vt_empty = vt_full + 2;  // [2] O MMA commit
  uint64_t* s_full = vt_empty + 2;   // [2] S MMA commit
  uint64_t* s_empty = s_full + 2;    // [2] O MMA commit (P read)
  uint64_t* p_full = s_empty + 2;    // [2] 8 softmax warps
  uint64_t* o_full = p_full + 2;     // [2] O MMA commit
  uint64_t* o_empty = o_full + 2;    // [2] 8 softmax warps
  uint64_t* pair_bar = o_empty + 2;  // [4] per TMEM lane quadrant: its 2 softmax warps
  uint64_t* mma_drain = pair_bar + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  float* rsum = reinterpret_cast<float*>(smem + L::kSumOff);
  auto give_up = [&](int wait_result, int code) {
    if (wait_result == tc::kWaitTimeout) tc::record_error(code);
    atomicExch(abort_flag, 1);
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = a.n_qt * a.B * a.H;

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_empty, 1);
    for (int s = 0; s < 2; s++) {
      tc::mbar_init(&k_full[s], 1);
      tc::mbar_init(&k_empty[s], a.fill_cache ? 2 : 1);
      tc::mbar_init(&vt_full[s], 2);
      tc::mbar_init(&vt_empty[s], 1);
      tc::mbar_init(&s_full[s], 1);
      tc::mbar_init(&s_empty[s], 1);
      tc::mbar_init(&p_full[s], 8);
      tc::mbar_init(&o_full[s], 1);
      tc::mbar_init(&o_empty[s], 8);
    }
    for (int i = 0; i < 4; i++) tc::mbar_init(&pair_bar[i], 2);
    tc::mbar_init(v_full, 1);
    tc::mbar_init(v_empty, 2);
    tc::mbar_init(mma_drain, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tm_q);
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM columns: S / P buffers at 0 and 128; O_j buffers at 256 and 256 + DH
  constexpr uint32_t kOCol = 256;

  grid_dep_launch();
  grid_dep_wait();  // q, k, v are the preceding kernel's outputs

  // Every role walks the same tiles (t = blockIdx.x, + gridDim.x, ...) and the
  // same key blocks; barrier phases follow the CTA-wide block counter g (and
  // the tile counter it for the Q buffer).
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int g = 0, it = 0;
      int gk = 0, gv = 0;  // K and V blocks whose copies were issued
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        const int w = tc::mbar_wait_or_abort(bar, parity, 2 * a.wait_ns, abort_flag);
        if (w != tc::kWaitOk) {
          give_up(w, tc::kErrTimeoutEmpty);
          ok = false;
        }
        return ok;
      };
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, it++) {
        const AttnTile tl = attn_tile(a, t);
        if (it >= 1 && !wait(q_empty, (it - 1) & 1)) break;
        tc::mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
        for (int c = 0; c < DH / 64; c++)
          tc::tma_load_4d(smem + L::kQOff + c * (kBQ * 128), &tm_q, 64 * c, tl.head, tl.q0, tl.seq, q_full);
        for (int j = 0; j < tl.nb; j++, g++) {
          const int s = g & 1;
          if (g >= 2 && !wait(&k_empty[s], ((g >> 1) - 1) & 1)) break;
          tc::mbar_arrive_expect_tx(&k_full[s], L::kKV);
#pragma unroll
          for (int c = 0; c < DH / 64; c++)
            tc::tma_load_4d(smem + L::kKOff + s * L::kKV + c * (kBK * 128), &tm_k, 64 * c, tl.head, j * kBK, tl.seq,
                            &k_full[s]);
          gk = g + 1;
          if (g >= 1 && !wait(v_empty, (g - 1) & 1)) break;
          tc::mbar_arrive_expect_tx(v_full, L::kKV);
#pragma unroll
          for (int c = 0; c < DH / 64; c++)
            tc::tma_load_4d(smem + L::kVOff + c * (kBK * 128), &tm_v, 64 * c, tl.head, j * kBK, tl.seq, v_full);
          gv = g + 1;
        }
      }
      // no copy into shared memory may be in flight when the CTA exits: the
      // last Q tile, the last two K blocks and the last V block issued
      if (it >= 1) tc::mbar_wait(q_full, (it - 1) & 1);
      for (int i = (gk > 2 ? gk - 2 : 0); i < gk; i++) tc::mbar_wait(&k_full[i & 1], (i >> 1) & 1);
      if (gv >= 1) tc::mbar_wait(v_full, (gv - 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16_f32(128, kBK);
      constexpr uint32_t idesc_o = tc::idesc_f16_f32(128, DH);
      const uint32_t qs = tc::smem_u32(smem + L::kQOff);
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity, int code) {
        if (!ok) return false;
        const int w = tc::mbar_wait_or_abort(bar, parity, a.wait_ns, abort_flag);
        if (w != tc::kWaitOk) {
          give_up(w, code);
          ok = false;
        }
        return ok;
      };
      auto issue_o = [&](int gi) {
        const int b = gi & 1;
        if (!wait(&p_full[b], (gi >> 1) & 1, tc::kErrTimeoutFull)) return;
        if (!wait(&vt_full[b], (gi >> 1) & 1, tc::kErrTimeoutFull)) return;
        if (gi >= 2 && !wait(&o_empty[b], ((gi >> 1) - 1) & 1, tc::kErrTimeoutAccum)) return;
        tc::tc_fence_after();
        const uint32_t vt = tc::smem_u32(smem + L::kVtOff + b * L::kKV);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++)
          tc::umma_f16_ta(tmem_base + kOCol + (uint32_t)(b * DH),
                          tmem_base + (uint32_t)(b * 128 + (kk >> 2) * 64 + (kk & 3) * 8),
                          tc::sdesc_k_sw128(vt + (kk >> 2) * (DH * 128) + (kk & 3) * 32), idesc_o, kk > 0 ? 1u : 0u);
        tc::umma_commit(&o_full[b]);
        tc::umma_commit(&s_empty[b]);
        tc::umma_commit(&vt_empty[b]);
      };
      int g = 0, it = 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, it++) {
        const AttnTile tl = attn_tile(a, t);
        if (!wait(q_full, it & 1, tc::kErrTimeoutFull)) break;
        for (int j = 0; j < tl.nb && ok; j++, g++) {
          const int b = g & 1;
          if (!wait(&k_full[b], (g >> 1) & 1, tc::kErrTimeoutFull)) break;
          if (g >= 2 && !wait(&s_empty[b], ((g >> 1) - 1) & 1, tc::kErrTimeoutAccum)) break;
          tc::tc_fence_after();
          const uint32_t ks = tc::smem_u32(smem + L::kKOff + b * L::kKV);
#pragma unroll
          for (int kk = 0; kk < DH / 16; kk++)
            tc::umma_f16(tmem_base + (uint32_t)(b * 128),
                         tc::sdesc_k_sw128(qs + (kk >> 2) * (kBQ * 128) + (kk & 3) * 32),
                         tc::sdesc_k_sw128(ks + (kk >> 2) * (kBK * 128) + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
          tc::umma_commit(&s_full[b]);
          tc::umma_commit(&k_empty[b]);
          if (j == tl.nb - 1) tc::umma_commit(q_empty);  // the tile's last product with Q
          if (j >= 1) issue_o(g - 1);
        }
        if (ok) issue_o(g - 1);
      }
      if (!ok) {
        // no MMA of this thread may still write tensor memory when it is freed
        tc::umma_commit(mma_drain);
        tc::mbar_wait(mma_drain, 0);
      }
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax + output
    const int qd = warp & 3;            // TMEM lane quadrant
    const int hf = (warp - 2) >> 2;     // half of the keys / of the output columns
    const int r = qd * 32 + lane;       // query row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    constexpr int OC = DH / 2;          // output columns of this thread
    bool ok = true;
    int pair_uses = 0;
    auto wait = [&](uint64_t* bar, uint32_t parity, int code) {
      const int w = tc::mbar_wait_or_abort(bar, parity, 2 * a.wait_ns, abort_flag);
      const bool all_ok = __all_sync(0xffffffffu, w == tc::kWaitOk);
      const bool any_timeout = __any_sync(0xffffffffu, w == tc::kWaitTimeout);
      if (!all_ok) {
        if (lane == 0) give_up(any_timeout ? tc::kWaitTimeout : tc::kWaitAborted, code);
        ok = false;
      }
      return all_ok;
    };
    // the quadrant's two warps meet (bounded: a partner that gave up never
    // leaves the other waiting); orders their shared-memory and TMEM accesses
    auto pair_sync = [&]() {
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&pair_bar[qd]);
      const bool met = wait(&pair_bar[qd], (uint32_t)(pair_uses & 1), tc::kErrTimeoutFull);
      pair_uses++;
      tc::tc_fence_after();
      return met;
    };
    float o[OC];
    auto accumulate = [&](int gi, float alpha) {
      const int b = gi & 1;
      if (!wait(&o_full[b], (gi >> 1) & 1, tc::kErrTimeoutAccum)) return;
      tc::tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < OC; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld_32x32b_x16(tmem_base + lane_off + kOCol + (uint32_t)(b * DH + hf * OC + c0),
                               *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        tc::tmem_ld_32x32b_x16(tmem_base + lane_off + kOCol + (uint32_t)(b * DH + hf * OC + c0 + 16),
                               *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; c++) o[c0 + c] = fmaf(o[c0 + c], alpha, __uint_as_float(v[c]));
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&o_empty[b]);
    };
    int g = 0;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      const AttnTile tl = attn_tile(a, t);
      const int qi = tl.q0 + r;
#pragma unroll
      for (int c = 0; c < OC; c++) o[c] = 0.0f;
      float m = -INFINITY, l = 0.0f;
      float alpha_prev = 0.0f;
      for (int j = 0; j < tl.nb && ok; j++, g++) {
        const int b = g & 1;
        if (!wait(&s_full[b], (g >> 1) & 1, tc::kErrTimeoutFull)) break;
        tc::tc_fence_after();
        // pass 1: this half's 64 scores (scaled, log2 domain; keys after the
        // query or past the sequence are -inf) -> row maximum
        const int kmax = min(qi, a.T - 1) - (j * kBK + hf * 64);  // keys e <= kmax are visible
        const uint32_t scol = tmem_base + lane_off + (uint32_t)(b * 128 + hf * 64);
        float mx = -INFINITY;
        {
          uint32_t sv[64];
          tc::tmem_ld_32x32b_x32(scol, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
          tc::tmem_ld_32x32b_x32(scol + 32u, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
          tc::tmem_ld_wait();
          // a tree, not a chain of 64 dependent maxima
          float m8[8];
#pragma unroll
          for (int u = 0; u < 8; u++) {
            float t = -INFINITY;
#pragma unroll
            for (int e = u; e < 64; e += 8)
              if (e <= kmax) t = fmaxf(t, __uint_as_float(sv[e]));
            m8[u] = t;
          }
          mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        }
        mx *= a.scale_log2;  // scale > 0: the maximum commutes with it
        float* rd = red + (g & 1) * (2 * kBQ);
        rd[hf * kBQ + r] = mx;
        if (!pair_sync()) break;  // both warps of this quadrant have written their maxima
        mx = fmaxf(rd[r], rd[kBQ + r]);
        const float m_new = fmaxf(m, mx);
        // a row with no visible key so far keeps m = -inf; its alpha is 1 and p 0
        const float alpha = m_new == -INFINITY ? 1.0f : tc::ex2_approx(m - m_new);
        const float msub = m_new == -INFINITY ? 0.0f : m_new;
        m = m_new;
        // pass 2: p = exp2(s - m) as f16 pairs along keys, written over this
        // half's own S columns (keys hf*64 + 16u .. +15 -> columns hf*64 + 8u ..
        // +7), which it has read already; the O product addresses its A slices
        // there.  32 scores per TMEM wait.
        float sum4[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four independent chains of additions
#pragma unroll
        for (int c = 0; c < 2; c++) {
          uint32_t sv[32];
          tc::tmem_ld_32x32b_x16(scol + (uint32_t)(32 * c), *reinterpret_cast<uint32_t(*)[16]>(&sv[0]));
          tc::tmem_ld_32x32b_x16(scol + (uint32_t)(32 * c + 16), *reinterpret_cast<uint32_t(*)[16]>(&sv[16]));
          tc::tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; e++) {
            const int k = 32 * c + 2 * e;
            const float x0 = k <= kmax ? fmaf(__uint_as_float(sv[2 * e]), a.scale_log2, -msub) : -INFINITY;
            const float x1 = k + 1 <= kmax ? fmaf(__uint_as_float(sv[2 * e + 1]), a.scale_log2, -msub) : -INFINITY;
            const float p0 = tc::ex2_approx(x0);
            const float p1 = tc::ex2_approx(x1);
            sum4[e & 3] += p0 + p1;
            const __half2 h2 = __floats2half2_rn(p0, p1);
            pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          tc::tmem_st_32x32b_x16(scol + (uint32_t)(16 * c), pk);
        }
        tc::tmem_st_wait();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&p_full[b]);
        l = fmaf(l, alpha, (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        if (j >= 1) accumulate(g - 1, alpha_prev);
        alpha_prev = alpha;
      }
      if (!ok) break;
      accumulate(g - 1, alpha_prev);
      if (!ok) break;
      // the row's sum is the two halves' sums (same running maximum)
      rsum[hf * kBQ + r] = l;
      if (!pair_sync()) break;
      const float lt = rsum[r] + rsum[kBQ + r];
      const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
      if (qi < a.T) {
        __half* op =
            a.out + (long long)tl.seq * a.o_seq + (long long)tl.head * a.o_head + (long long)qi * a.o_pos + hf * OC;
#pragma unroll
        for (int c = 0; c < OC; c += 8) {
          uint4 w;
          __half2 h0 = __floats2half2_rn(o[c] * inv, o[c + 1] * inv);
          __half2 h1 = __floats2half2_rn(o[c + 2] * inv, o[c + 3] * inv);
          __half2 h2 = __floats2half2_rn(o[c + 4] * inv, o[c + 5] * inv);
          __half2 h3 = __floats2half2_rn(o[c + 6] * inv, o[c + 7] * inv);
          w.x = *reinterpret_cast<uint32_t*>(&h0);
          w.y = *reinterpret_cast<uint32_t*>(&h1);
          w.z = *reinterpret_cast<uint32_t*>(&h2);
          w.w = *reinterpret_cast<uint32_t*>(&h3);
          *reinterpret_cast<uint4*>(op + c) = w;
        }
        if (a.lse && hf == 0)
          a.lse[((long long)tl.seq * a.H + tl.head) * a.T + qi] =
              (m + __log2f(lt > 0.0f ? lt : 1e-30f)) * 0.69314718f;
      }
    }
  } else {
    // ------------------------------------------------------------ V transposers
    // V block [128 keys][DH] (boxes of 64 columns, 128-byte rows, 128-byte
    // swizzle) -> V^T [DH rows][128 keys] (two boxes of 64 keys, same swizzle).
    // Lane 8i + k of an x4 ldmatrix.trans / stmatrix pair handles row k of 8x8
    // block i; a warp takes blocks (key group kb, column group cb) in turn.
    const int tw = warp - 10;
    constexpr int kBlocks = (kBK / 8) * (DH / 8);
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      const AttnTile tl = attn_tile(a, t);
      for (int j = 0; j < tl.nb; j++, g++) {
        const int s = g & 1;
        int w = tc::mbar_wait_or_abort(v_full, g & 1, 2 * a.wait_ns, abort_flag);
        if (w == tc::kWaitOk && g >= 2)
          w = tc::mbar_wait_or_abort(&vt_empty[s], ((g >> 1) - 1) & 1, 2 * a.wait_ns, abort_flag);
        const bool all_ok = __all_sync(0xffffffffu, w == tc::kWaitOk);
        if (!all_ok) {
          if (lane == 0)
            give_up(__any_sync(0xffffffffu, w == tc::kWaitTimeout) ? tc::kWaitTimeout : tc::kWaitAborted,
                    tc::kErrTimeoutEmpty);
          ok = false;
          break;
        }
        const uint8_t* vsrc = smem + L::kVOff;
        uint8_t* vdst = smem + L::kVtOff + s * L::kKV;
        const int mi = lane >> 3, k8 = lane & 7;
        for (int blk = tw * 4; blk < kBlocks; blk += 8) {
          // four blocks blk .. blk + 3: key group kb, column groups cb .. cb + 3
          const int kb = blk / (DH / 8), cb = (blk % (DH / 8)) + mi;
          const int key = kb * 8 + k8, col = cb * 8;
          const uint32_t src = tc::smem_u32(vsrc + (col >> 6) * (kBK * 128) + key * 128 +
                                            ((((col & 63) >> 3) ^ (key & 7)) << 4));
          uint32_t r0, r1, r2, r3;
          tc::ldmatrix_x4_trans(src, r0, r1, r2, r3);
          // r[i] now holds the fragment of block i's transpose (rows = columns of V)
          const int vrow = cb * 8 + k8;  // lane 8i + k8 stores row k8 of transposed block i
          const int kk = kb * 8;         // its 8 keys
          const uint32_t dst = tc::smem_u32(vdst + (kk >> 6) * (DH * 128) + vrow * 128 +
                                            ((((kk & 63) >> 3) ^ (vrow & 7)) << 4));
          tc::stmatrix_x4(dst, r0, r1, r2, r3);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&vt_full[s]);
        if (tw == 0 && lane == 0) {
          // KV-cache fill: the block's K and V boxes go to the caches once, from
          // the CTA whose query tile is the block's own (its diagonal block);
          // the shared-memory buffers are released only after TMA has read them
          if (a.fill_cache && j == tl.nb - 1) {
            bool kok = tc::mbar_wait_or_abort(&k_full[s], (g >> 1) & 1, 2 * a.wait_ns, abort_flag) == tc::kWaitOk;
            if (kok) {
#pragma unroll
              for (int c = 0; c < DH / 64; c++) {
                tc::tma_store_4d(&tm_kc, 64 * c, tl.head, j * kBK, tl.seq, smem + L::kKOff + s * L::kKV + c * (kBK * 128));
                tc::tma_store_4d(&tm_vc, 64 * c, tl.head, j * kBK, tl.seq, smem + L::kVOff + c * (kBK * 128));
              }
              tc::bulk_commit();
              tc::bulk_wait_read<0>();
            } else {
              give_up(tc::kWaitAborted, tc::kErrTimeoutEmpty);
            }
          }
          if (a.fill_cache) tc::mbar_arrive(&k_empty[s]);
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(v_empty);
      }
    }
    if (tw == 0 && lane == 0 && a.fill_cache) tc::bulk_wait_all();  // the cache writes are complete
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*AttnEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static AttnEncodeFn attn_encode_fn() {
  static AttnEncodeFn fn = []() -> AttnEncodeFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<AttnEncodeFn>(p);
  }();
  return fn;
}

// 4-D view {DH, H, T, B} of q, k or v (element strides s_head, s_pos, s_seq),
// boxes of [1 sequence][128 positions][1 head][64 columns], 128-byte swizzle.
static bool attn_tmap(CUtensorMap* tm, const __half* base, int DH, int H, int T, int B, long long s_head,
                      long long s_pos, long long s_seq) {
  AttnEncodeFn enc = attn_encode_fn();
  if (!enc) return false;
  const cuuint64_t dim[4] = {(cuuint64_t)DH, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t str[3] = {(cuuint64_t)s_head * 2, (cuuint64_t)s_pos * 2, (cuuint64_t)s_seq * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)kBK, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(base), dim, str, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kAttnMaxDevices = 64;

template <int DH>
static cudaError_t launch_attn_t(const __half* q, const __half* k, const __half* v, long long s_head, long long s_pos,
                                 long long s_seq, int B, int H, int T, float scale, __half* out, long long o_seq,
                                 long long o_head, long long o_pos, float* lse, __half* k_cache, __half* v_cache,
                                 int max_seq, cudaStream_t st, unsigned long long wait_ns) {
  using L = AttnSmem<DH>;
  CUtensorMap tq, tk, tv, tkc, tvc;
  if (!attn_tmap(&tq, q, DH, H, T, B, s_head, s_pos, s_seq) || !attn_tmap(&tk, k, DH, H, T, B, s_head, s_pos, s_seq) ||
      !attn_tmap(&tv, v, DH, H, T, B, s_head, s_pos, s_seq))
    return cudaErrorInvalidValue;
  // the caches [B][max_seq][H * DH]: positions 0 .. T - 1 written (the map's
  // extent clips the rest of a partial block)
  const bool fill = k_cache != nullptr && v_cache != nullptr;
  memset(&tkc, 0, sizeof(tkc));
  memset(&tvc, 0, sizeof(tvc));
  if (fill) {
    const long long d = (long long)H * DH;
    if (!attn_tmap(&tkc, k_cache, DH, H, T, B, DH, d, (long long)max_seq * d) ||
        !attn_tmap(&tvc, v_cache, DH, H, T, B, DH, d, (long long)max_seq * d))
      return cudaErrorInvalidValue;
  }
  auto kern = attn_prefill_kernel<DH>;
  static bool attr_set[kAttnMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kAttnMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  AttnArgs a;
  a.T = T; a.H = H; a.B = B;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out; a.o_seq = o_seq; a.o_head = o_head; a.o_pos = o_pos;
  a.lse = lse;
  a.n_qt = (T + kBQ - 1) / kBQ;
  a.wait_ns = wait_ns;
  a.fill_cache = fill ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  int dev_sms = 148;
  cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (long long)a.n_qt * B * H;
  cfg.gridDim = dim3((unsigned)(tiles < dev_sms ? tiles : dev_sms));  // persistent: one CTA per SM
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, tkc, tvc, a);
}

// Causal attention of B sequences x H heads over T positions, head size DH (64
// or 128): q / k / v element (seq, head, pos, i) at base + seq s_seq + head
// s_head + pos s_pos + i, out likewise with its own strides, lse (optional)
// [B][H][T]; with k_cache and v_cache ([B][max_seq][H * DH], optional) the
// keys and values of positions 0 .. T - 1 are also written there.
cudaError_t launch_attention_prefill(const __half* q, const __half* k, const __half* v, int DH, long long s_head,
                                     long long s_pos, long long s_seq, int B, int H, int T, float scale, __half* out,
                                     long long o_seq, long long o_head, long long o_pos, float* lse,
                                     __half* k_cache, __half* v_cache, int max_seq, cudaStream_t st) {
  if (DH == 64)
    return launch_attn_t<64>(q, k, v, s_head, s_pos, s_seq, B, H, T, scale, out, o_seq, o_head, o_pos, lse, k_cache,
                             v_cache, max_seq, st, tc::kWaitLimitNs);
  if (DH == 128)
    return launch_attn_t<128>(q, k, v, s_head, s_pos, s_seq, B, H, T, scale, out, o_seq, o_head, o_pos, lse, k_cache,
                              v_cache, max_seq, st, tc::kWaitLimitNs);
  return cudaErrorInvalidValue;
}

// Reads and clears this unit's device error flag (synchronous).
int attn_take_device_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) cudaMemcpyToSymbol(tc::g_device_error, &zero, sizeof(int));
  return v;
}

}  // namespace aria_q4
