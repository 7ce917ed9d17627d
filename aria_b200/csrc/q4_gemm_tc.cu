// q4_gemm_tc.cu -- prefill-regime Q4_0 projection on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Replaces, for Q4_0 weights and M > 32 tokens, the cuBLAS fp16 GEMM of
// lold3344/ARIA's forward pass (`gemm()` src/transformer_cuda.rs:615-640 at
// :1583, :1686, :1753, :1805, :1864), which there runs with M = t tokens
// (forward_gpu recomputes the whole prompt every step).
//
// Persistent kernel: one CTA per SM walks the output tiles D[128 weight rows][BT
// tokens] = W_tile[128 x K] . X_tile[BT x K]^T ("swap AB": the weights are the
// 128-row UMMA operand, so each dequantised weight serves BT = up to 256 tokens).
// Fourteen warps, specialised:
//   warp 8      TMA producer: X tiles [BT x 128 k] f16 per stage (two 64-k boxes,
//               128-byte swizzle, no multicast)
//   warps 0-7   dequantisers, two warpgroups taking alternate 128-k groups (one
//               stage each): one weight row per thread; the row's codes are streamed
//               with cp.async into a shared-memory ring several groups ahead, turned into (q-8)*scale f16
//               (LOP3/HSUB/HMUL) and written with tcgen05.st straight into tensor
//               memory, where the MMA reads its A operand: the dequantised weights
//               never cost shared-memory bandwidth (which X tiles alone keep near
//               its 128 B/clk limit)
//   warp 9      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BT, K=16,
//               A from TMEM, B = X tile from shared memory, f32 accumulator in TMEM);
//               tcgen05.commit releases operand stages and
//               hands finished accumulators to the epilogue
//   warp 14     (64-token tiles only) a second issuer: it takes the stages of
//               dequant warpgroup 1 into a second accumulator, which the
//               epilogue adds to the first
//   warps 10-13 epilogue: tcgen05.ld of one of two TMEM accumulators (so the next
//               tile's MMAs overlap this tile's stores), alpha/bias/beta, f16/f32 store
// Operand stages (128 k: one code group) are an mbarrier ring (STAGES deep); the
// accumulators have their own full/empty barriers.  A stage of 128 k rather
// than 64 k halves the barrier waits, fences and commits the single MMA-issuing
// thread performs per MMA -- that thread's issue latency bounds the pipe.  Every wait is bounded (one second); on expiry
// the kernel records an error code in g_device_error, unwinds, frees its TMEM
// and returns instead of hanging the GPU.
//
// The dequantised weight is rounded once to f16 ((q-8)*scale, relative error
// <= 2^-11 per weight); products and sums are f32 in the tensor core.
#include <cuda.h>

#include <cstring>

#include "q4_common.cuh"
#include "q4_tcgen05.cuh"

namespace aria_q4 {

struct TcArgs {
  const uint8_t* qs;
  const __half* scales;
  int K, N, Kp, M;
  void* y;
  int ydt, ldy;
  const __half* bias;
  float alpha, beta;
  // split-K: every output tile is computed as `splits` K-slices (work units);
  // each unit's f32 partial goes to ws_part, and the last unit of a tile to
  // finish (counted per tile and TMEM lane quadrant in ws_cnt, which every call
  // leaves zero) adds the partials in slice order and writes the output.
  int splits;
  float* ws_part;
  unsigned* ws_cnt;
  // limit of the MMA issuer's waits (tc::kWaitLimitNs in production); every
  // other wait (producers, epilogue), which depends on the issuer's progress,
  // gets twice as long, so a stalled operand stage is reported by the issuer
  unsigned long long wait_ns;
  // failure-path test only: the X-tile producer issues no copies, so the MMA
  // issuer's first wait runs out and the CTA unwinds
  int no_x_loads;
  // the weights are not written by the preceding kernel on the stream: the
  // dequantisers may load and dequantise them before that kernel completes
  int const_weights;
  // epilogue of unsplit tiles: 0 = per-thread stores (any output), else
  // outputs staged in shared memory and written by TMA: kEpiStore (beta = 0)
  // or kEpiAdd (beta = 1: a TMA add-reduction into y, no loads of old values)
  int tma_epi;
};
enum : int { kEpiThreads = 0, kEpiStore = 1, kEpiAdd = 2 };

// K-slice of work unit `unit` in 128-k groups: [g0, g1)
__device__ __forceinline__ void tc_unit(const TcArgs& a, int unit, int KG, int& tile, int& split, int& g0, int& g1) {
  tile = unit / a.splits;
  split = unit - tile * a.splits;
  g0 = split * KG / a.splits;
  g1 = (split + 1) * KG / a.splits;
}

constexpr int kTcThreads = 448;  // 8 dequant + TMA + MMA + 4 epilogue warps
constexpr int kBK = 64;         // k per TMA box (one 128-byte swizzle row of f16)
constexpr int kStageK = 128;    // k per pipeline stage: one 128-k code group, two TMA boxes
constexpr int kAStageCols = 64;  // TMEM columns of one dequantised A stage: 128 rows x 128 k f16

constexpr int kQDepth = 4;  // 128-k code groups in flight per dequant warpgroup
// per warpgroup and ring slot: each row's whole 64-byte code group (128 rows) and
// its scales (NK: 8 B per row; KN: 256 B per 32-row group)
constexpr int kQSlot = 128 * 64;
constexpr int kSSlot = 128 * 8 > 4 * 256 ? 128 * 8 : 4 * 256;
// staged epilogue: per epilogue warp, one 2-KB box of [32 tokens][32 rows] f16
// or [16 tokens][32 rows] f32
constexpr int kEChunk = 1024;  // the box is two of these

template <int BT, int STAGES>
struct TcSmem {
  static constexpr int kXTile = BT * kBK * 2;  // one TMA box [BT x 64 k]
  static constexpr int kStage = 2 * kXTile;     // one 128-k stage
  static constexpr int kQOff = STAGES * kStage;
  static constexpr int kSOff = kQOff + 2 * kQDepth * kQSlot;
  static constexpr int kEOff = kSOff + 2 * kQDepth * kSSlot;  // epilogue staging, 1024-aligned
  static constexpr int kBarOff = kEOff + 4 * 2 * kEChunk;
  static constexpr int kBytes = kBarOff + 512 + 1024;  // barriers + alignment slack
};

__device__ __forceinline__ void cp_async_16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tc::smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(tc::smem_u32(dst)), "l"(src), "r"(valid ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tc::smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// v[i] += u[i] as f32 (the two issuers' accumulators of one unit)
template <int N>
__device__ __forceinline__ void add_f32_regs(uint32_t (&v)[N], const uint32_t (&u)[N]) {
#pragma unroll
  for (int i = 0; i < N; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) + __uint_as_float(u[i]));
}

// ISS MMA-issuing threads (warp 9, and warp 14 when ISS = 2).  One thread
// issues a tcgen05.mma about every 67 cycles whatever N, while a 128 x 64 x 16
// MMA holds 32 cycles of tensor work; two threads issuing into separate
// accumulators reach one MMA per ~37 cycles (measured on B200, back-to-back
// MMAs).  With ISS = 2, issuer w takes the 128-k groups of dequant warpgroup w
// (G % 2 == w) into its own accumulator, and the epilogue adds the two.
template <int LAYOUT, int BT, int STAGES, int NACC, int ISS>
__global__ void __launch_bounds__(kTcThreads + 32 * (ISS - 1), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                   const TcArgs a, int n_tiles, int num_tiles) {
  using L = TcSmem<BT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // TMEM: NACC f32 accumulators [128 x BT], then kASlots dequantised A stages.
  // Every free TMEM column holds A stages (up to 12): each dequant warpgroup's
  // sub-ring depth bounds how many stages are in flight between dequantisation
  // and MMA completion, which sets the stage rate when few tokens make each
  // MMA short (measured: 64 stages per tile at BT = 64 ran at ~600 cycles each
  // with four slots in all)
  // NACC = 2 accumulators let the next tile's MMAs overlap this tile's
  // epilogue; NACC = 1 leaves TMEM room for token tiles up to 256 (for shapes
  // whose tiles fit one round of CTAs there is no next tile to overlap).  With
  // BT = 192 and NACC = 2 one A slot per warpgroup remains: a warpgroup then
  // dequantises group G + 2 while the MMAs of the other warpgroup's group G + 1
  // run, which at 192 tokens take longer than the dequantisation.
  static_assert(ISS == 1 || ISS == 2, "one or two MMA issuers");
  constexpr int kAccCols = NACC * ISS * BT;  // accumulator buf, issuer w at column (buf * ISS + w) * BT
  constexpr int kFreeCols = 512 - kAccCols;
  constexpr int kASlots = kFreeCols / kAStageCols >= 8 ? 8 : (kFreeCols / kAStageCols) & ~1;
  static_assert(kASlots >= 2, "one A slot per dequant warpgroup at least");
  constexpr int kAPer = kASlots / 2;
  constexpr uint32_t kAColBase = kAccCols;  // A stages follow the accumulators
  constexpr uint32_t kNeed = kAccCols + kASlots * kAStageCols;
  constexpr uint32_t kCols = kNeed <= 32 ? 32 : kNeed <= 64 ? 64 : kNeed <= 128 ? 128 : kNeed <= 256 ? 256 : 512;
  static_assert(kNeed <= 512, "TMEM budget");
  static_assert(kAColBase + kASlots * kAStageCols <= kCols, "A stages inside the allocation");
  // X tiles: one ring indexed by the CTA's stage counter (producer and MMA walk it
  // in order).  Dequantised A stages: two private sub-rings of kASlots/2, one per
  // dequant warpgroup, indexed by that warpgroup's own stage counter -- so no
  // waiter can fall two phases behind a barrier whose slot another warpgroup uses.
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty_x = full_x + STAGES;
  uint64_t* full_a = empty_x + STAGES;   // [kASlots]
  uint64_t* empty_a = full_a + kASlots;  // [kASlots]
  uint64_t* acc_full = empty_a + kASlots;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* mma_drain = acc_empty + 2;     // [ISS] error path: completion of every issued MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + ISS);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  // A wait that runs out records its code and raises abort_flag; every other
  // wait of the CTA then returns at once (its phase can no longer complete),
  // so the CTA unwinds within one wait limit.
  auto give_up = [&](int wait_result, int code) {
    if (wait_result == tc::kWaitTimeout) tc::record_error(code);
    atomicExch(abort_flag, 1);
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = (num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full_x[s], 1);
      tc::mbar_init(&empty_x[s], 1);
    }
    for (int s = 0; s < kASlots; s++) {
      tc::mbar_init(&full_a[s], 4);  // one arrival per dequant warp
      tc::mbar_init(&empty_a[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      tc::mbar_init(&acc_full[b], ISS);  // one commit per issuer
      tc::mbar_init(&acc_empty[b], 4);   // one arrival per epilogue warp
    }
    for (int w = 0; w < ISS; w++) tc::mbar_init(&mma_drain[w], 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, kCols);
    tc::tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tc::prefetch_tmap(&tmap_x);
    if (a.tma_epi != kEpiThreads) tc::prefetch_tmap(&tmap_y);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  grid_dep_launch();
  // Programmatic dependent launch: the X tiles, the outputs (and, with split-K,
  // the workspace) may be written or read by the preceding kernel, so the X
  // producer, the MMA issuer and the epilogue wait for it to complete.  The
  // weights are constants when the caller says so: the dequantisers then fill
  // the first A stages of tensor memory while that kernel drains (their waits
  // for free stages, bounded at twice the limit, then include its tail).
  if (!a.const_weights || warp >= 8) grid_dep_wait();

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && !a.no_x_loads) {
      int it = 0;
      bool ok = true;
      const int KG = a.Kp >> 7;
      for (int j = 0; j < my_tiles && ok; j++) {
        int tile, split, g0, g1;
        tc_unit(a, blockIdx.x + j * gridDim.x, KG, tile, split, g0, g1);
        const int m0 = (tile / n_tiles) * BT;
        for (int G = g0; G < g1; G++, it++) {
          const int s = it % STAGES;
          if (it >= STAGES) {
            const int w = tc::mbar_wait_or_abort(&empty_x[s], ((it / STAGES) - 1) & 1, 2 * a.wait_ns, abort_flag);
            if (w != tc::kWaitOk) {
              give_up(w, tc::kErrTimeoutEmpty);
              ok = false;
              break;
            }
          }
          // two boxes of 64 k on one barrier (the second may lie past K: zero-filled)
          tc::mbar_arrive_expect_tx(&full_x[s], 2 * L::kXTile);
          tc::tma_load_2d(smem + s * L::kStage, &tmap_x, G * kStageK, m0, &full_x[s]);
          tc::tma_load_2d(smem + s * L::kStage + L::kXTile, &tmap_x, G * kStageK + kBK, m0, &full_x[s]);
        }
      }
      // never leave the CTA while a copy into its shared memory is in flight
      for (int i = (it > STAGES ? it - STAGES : 0); i < it; i++)
        tc::mbar_wait(&full_x[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 9 || (ISS == 2 && warp == 14)) {
    // ------------------------------------------------------------ MMA issuer(s)
    const int iw = warp == 9 ? 0 : 1;  // issuer index
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(128, BT);
      // The issuing thread's per-stage work is the MMA pipe's throughput limit
      // (every tcgen05 and mbarrier operation costs tens of cycles of issue
      // latency), so ring positions advance incrementally and descriptors are
      // derived from one precomputed base: no divisions or descriptor
      // rebuilding inside the loop.
      const uint64_t desc0 = tc::sdesc_k_sw128(tc::smem_u32(smem));  // X slot 0; address field in 16-B units
      int xslot = 0;
      uint32_t xph = 0;
      int aslot0 = 0, aslot1 = 0;  // position in each warpgroup's A sub-ring
      uint32_t aph0 = 0, aph1 = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; j++) {
        const int buf = NACC == 2 ? (j & 1) : 0;
        const int use = NACC == 2 ? (j >> 1) : j;  // earlier uses of this accumulator
        if (use >= 1) {
          const int w = tc::mbar_wait_or_abort(&acc_empty[buf], (use - 1) & 1, a.wait_ns, abort_flag);
          if (w != tc::kWaitOk) {
            give_up(w, tc::kErrTimeoutAccum);
            ok = false;
            break;
          }
        }
        tc::tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)((buf * ISS + iw) * BT);
        int tile, split, g0, g1;
        tc_unit(a, blockIdx.x + j * gridDim.x, a.Kp >> 7, tile, split, g0, g1);
#pragma unroll 2
        for (int G = g0; G < g1; G++) {
          const int w = G & 1;  // warpgroup that dequantised this stage
          if (ISS == 2 && w != iw) {  // the other issuer's stage: only keep the X ring position
            if (++xslot == STAGES) { xslot = 0; xph ^= 1u; }
            continue;
          }
          const int as = w ? kAPer + aslot1 : aslot0;
          const uint32_t aph = w ? aph1 : aph0;
          if (w) {
            if (++aslot1 == kAPer) { aslot1 = 0; aph1 ^= 1u; }
          } else {
            if (++aslot0 == kAPer) { aslot0 = 0; aph0 ^= 1u; }
          }
          int wr = tc::mbar_wait_or_abort(&full_x[xslot], xph, a.wait_ns, abort_flag);
          if (wr == tc::kWaitOk) wr = tc::mbar_wait_or_abort(&full_a[as], aph, a.wait_ns, abort_flag);
          if (wr != tc::kWaitOk) {
            give_up(wr, tc::kErrTimeoutFull);
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint64_t bdesc = desc0 + (uint64_t)((uint32_t)(xslot * L::kStage) >> 4);
          const uint32_t at = tmem_base + kAColBase + (uint32_t)(as * kAStageCols);
          // eight K = 16 slices: slice kk reads box kk / 4 at byte 32 * (kk % 4)
#pragma unroll
          for (int kk = 0; kk < kStageK / 16; kk++)
            tc::umma_f16_ta(tmem_d, at + (uint32_t)(kk * 8),
                            bdesc + (uint64_t)(((kk >> 2) * L::kXTile + (kk & 3) * 32) >> 4), idesc,
                            (G >= g0 + ISS || kk > 0) ? 1u : 0u);
          tc::umma_commit(&empty_x[xslot]);
          tc::umma_commit(&empty_a[as]);
          if (++xslot == STAGES) { xslot = 0; xph ^= 1u; }
        }
        tc::umma_commit(&acc_full[buf]);  // also on the error path, so the epilogue is released
      }
      if (!ok) {
        // no MMA issued by this thread may still write tensor memory when the CTA
        // frees it: wait (bounded) for all of them
        tc::umma_commit(&mma_drain[iw]);
        tc::mbar_wait(&mma_drain[iw], 0);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ dequantisers
    // Two warpgroups: WG w (warps 4w..4w+3) owns the 128-k groups G = w, w+2, ...
    // of every tile and feeds their 128-k stages.  Each thread owns one
    // weight row (= TMEM lane); each warp streams its 32 rows' 64-byte code
    // groups plus their scales into a kQDepth-deep shared-memory ring with
    // 16-byte cp.async, so loads run groups ahead without holding registers; the
    // four 16-byte chunks of a row are stored XOR-swizzled by (row >> 1) & 3 so
    // neighbouring rows' 128-bit reads hit distinct banks.  KN scales (one per k for a 32-row
    // group) are shared by a warp: lanes 0..15 copy the group's 256 bytes.
    const int wg = warp >> 2;         // 0 or 1
    const int wl = warp & 3;          // warp within the warpgroup = TMEM lane quadrant
    const int r = threadIdx.x & 127;  // weight row of the tile = TMEM lane
    const int sw = (r >> 1) & 3;
    const size_t RB = (size_t)a.Kp >> 1;
    const int KG = a.Kp >> 7;
    uint8_t* qring = smem + L::kQOff + wg * kQDepth * kQSlot;
    uint8_t* sring = smem + L::kSOff + wg * kQDepth * kSSlot;
    // This warpgroup's groups, in order: for each of the CTA's work units, the
    // groups G of its K-slice with G % 2 == wg.  Two cursors walk the sequence:
    // the copy issuer (kQDepth - 1 groups ahead) and the dequantiser.
    struct Cursor {
      int j, tile, g1, G;
    };
    auto cursor_first = [&](Cursor& c, int j) {
      c.j = j;
      c.G = 1 << 30;
      for (; c.j < my_tiles; c.j++) {
        int split, g0;
        tc_unit(a, blockIdx.x + c.j * gridDim.x, KG, c.tile, split, g0, c.g1);
        c.G = g0 + ((g0 & 1) != wg ? 1 : 0);
        if (c.G < c.g1) return;
      }
    };
    auto cursor_next = [&](Cursor& c) {
      c.G += 2;
      if (c.G >= c.g1) cursor_first(c, c.j + 1);
    };
    Cursor ic;
    cursor_first(ic, 0);
    int iseq = 0;
    auto issue = [&]() {
      const int slot = iseq % kQDepth;
      iseq++;
      if (ic.j < my_tiles) {
        const int G = ic.G;
        const int nb = (ic.tile % n_tiles) * 128;
        // codes: the warp copies its 32 rows cooperatively, lane l taking 16-byte
        // chunk l % 4 of row 8u + l / 4, so one copy instruction reads eight whole
        // 64-byte row segments (instead of 32 scattered 16-byte pieces)
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int rl = 32 * wl + 8 * u + (lane >> 2);
          const int q = lane & 3;
          const int nr = nb + rl;
          const bool okr = nr < a.N;
          cp_async_16(qring + slot * kQSlot + rl * 64 + ((q ^ ((rl >> 1) & 3)) << 4),
                      a.qs + (okr ? (size_t)nr : 0) * RB + (size_t)G * 64 + 16 * q, okr);
        }
        const int n = nb + r;
        const bool ok_row = n < a.N;
        const size_t nn = ok_row ? (size_t)n : 0;
        if (LAYOUT == 1) {
          cp_async_8(sring + slot * kSSlot + r * 8, a.scales + ((size_t)G * a.N + nn) * 4, ok_row);
        } else if (lane < 16) {
          const int grp = (nb + wl * 32) >> 5;
          const bool ok_grp = grp * 32 < a.N;
          const __half* ssrc = a.scales + (size_t)(ok_grp ? grp : 0) * a.Kp + (size_t)G * 128 + lane * 8;
          cp_async_16(sring + slot * kSSlot + wl * 256 + lane * 16, ssrc, ok_grp);
        }
        cursor_next(ic);
      }
      cp_async_commit();  // an empty group keeps the wait count uniform
    };
#pragma unroll
    for (int p = 0; p < kQDepth - 1; p++) issue();
    bool ok = true;
    int seq = 0;
    int acnt = 0;  // stages this warpgroup has produced into its A sub-ring
    Cursor dc;
    for (cursor_first(dc, 0); dc.j < my_tiles && ok; cursor_next(dc), seq++) {
      {
        __syncwarp();  // every lane is done reading the slot the next issue overwrites
        issue();
        cp_async_wait<kQDepth - 1>();  // group `seq` has landed for this thread
        __syncwarp();                  // ... and for the warp's shared KN scale row
        const int slot = seq % kQDepth;
        const uint8_t* qsrc = qring + slot * kQSlot + r * 64;
        uint4 gq[4];
#pragma unroll
        for (int q = 0; q < 4; q++) gq[q] = *reinterpret_cast<const uint4*>(qsrc + ((q ^ sw) << 4));
        const uint2 gs = (LAYOUT == 1) ? *reinterpret_cast<const uint2*>(sring + slot * kSSlot + r * 8)
                                       : make_uint2(0, 0);
        const uint8_t* kscale = sring + slot * kSSlot + wl * 256;
        const int c = acnt++;
        const int s = wg * kAPer + c % kAPer;  // A slot in this warpgroup's sub-ring
        // warp-uniform outcome: tcgen05.st and the per-warp arrival below are warp-collective
        if (c >= kAPer) {
          const int w = tc::mbar_wait_or_abort(&empty_a[s], ((c / kAPer) - 1) & 1, 2 * a.wait_ns, abort_flag);
          const bool all_ok = __all_sync(0xffffffffu, w == tc::kWaitOk);
          const bool any_timeout = __any_sync(0xffffffffu, w == tc::kWaitTimeout);
          if (!all_ok) {
            if (lane == 0) give_up(any_timeout ? tc::kWaitTimeout : tc::kWaitAborted, tc::kErrTimeoutEmpty);
            ok = false;
            break;
          }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
          // word (t, 2h+ii) holds local k = 64h + 32*ii + 8t .. +7, i.e. TMEM
          // columns 32h + 16*ii + 4t .. +3 of the stage
          uint32_t av[32];
#pragma unroll
          for (int t = 0; t < 4; t++) {
#pragma unroll
            for (int ii = 0; ii < 2; ii++) {
              const int i = 2 * h + ii;
              const uint32_t w = (i == 0) ? gq[t].x : (i == 1) ? gq[t].y : (i == 2) ? gq[t].z : gq[t].w;
              uint32_t d[4];
              dequant_word_f16x2(w, d);
              if (LAYOUT == 1) {
                const uint32_t swd = (i < 2) ? gs.x : gs.y;
                const uint32_t s1 = (i & 1) ? (swd >> 16) : (swd & 0xFFFFu);
                const uint32_t s2 = s1 | (s1 << 16);
#pragma unroll
                for (int e = 0; e < 4; e++) d[e] = hmul2_u32(d[e], s2);
              } else {
                const uint4 s8 = *reinterpret_cast<const uint4*>(kscale + (32 * i + 8 * t) * 2);
                d[0] = hmul2_u32(d[0], s8.x);
                d[1] = hmul2_u32(d[1], s8.y);
                d[2] = hmul2_u32(d[2], s8.z);
                d[3] = hmul2_u32(d[3], s8.w);
              }
#pragma unroll
              for (int e = 0; e < 4; e++) av[16 * ii + 4 * t + e] = d[e];
            }
          }
          tc::tmem_st_32x32b_x32(
              tmem_base + ((uint32_t)(32 * wl) << 16) + kAColBase + (uint32_t)(s * kAStageCols + 32 * h), av);
        }
        tc::tmem_st_wait();
        tc::tc_fence_before();
        __syncwarp();  // the warp's 32 lanes have stored: one arrival for the warp
        if (lane == 0) tc::mbar_arrive(&full_a[s]);
      }
    }
    cp_async_wait<0>();  // no copy into shared memory may outlive the loop
  } else {
    // ------------------------------------------------------------ epilogue (warps 10..13)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int rr = q * 32 + lane;
    const int KG = a.Kp >> 7;
    // 32 outputs of one row n, tokens tok0 .. tok0 + ntok - 1 (stride ldy), through
    // store_outputs: the activation, every old value for the beta term loaded
    // (unconditionally: masked tokens read the last valid one) before the first
    // store, then the stores
    auto store32 = [&](int tok0, int ntok, int n, float (&o)[32]) {
      store_outputs<32>(
          a.y, a.ydt, o, a.beta, [&](int jj) { return (size_t)(tok0 + min(jj, ntok - 1)) * a.ldy + n; },
          [&](int jj) { return jj < ntok; });
    };
    for (int j = 0; j < my_tiles; j++) {
      const int buf = NACC == 2 ? (j & 1) : 0;
      const int use = NACC == 2 ? (j >> 1) : j;
      int tile, split, g0, g1;
      tc_unit(a, blockIdx.x + j * gridDim.x, KG, tile, split, g0, g1);
      const int n = (tile % n_tiles) * 128 + rr;
      const int m0 = (tile / n_tiles) * BT;
      // warp-uniform decisions: the per-warp arrival below is reached by all lanes or none
      {
        const int w = tc::mbar_wait_or_abort(&acc_full[buf], use & 1, 2 * a.wait_ns, abort_flag);
        const bool all_ok = __all_sync(0xffffffffu, w == tc::kWaitOk);
        const bool any_timeout = __any_sync(0xffffffffu, w == tc::kWaitTimeout);
        if (!all_ok) {
          if (lane == 0) give_up(any_timeout ? tc::kWaitTimeout : tc::kWaitAborted, tc::kErrTimeoutAccum);
          break;
        }
      }
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(abort_flag) != 0)) break;
      tc::tc_fence_after();
      const bool row_ok = n < a.N;
      const float bias = (a.bias && row_ok) ? __half2float(a.bias[n]) : 0.0f;
      // accumulators of this unit: with two issuers, issuer w's holds the groups
      // G % 2 == w (absent when the unit has a single group of the other parity);
      // the epilogue reads the first present one and adds the second
      const uint32_t tmem_d0 = tmem_base + (uint32_t)(buf * ISS * BT) + ((uint32_t)(q * 32) << 16);
      const bool has0 = ISS == 1 || g1 - g0 >= 2 || (g0 & 1) == 0;
      const bool add2 = ISS == 2 && has0 && g1 - g0 >= 2;
      const uint32_t tmem_d = has0 ? tmem_d0 : tmem_d0 + (uint32_t)BT;
      const uint32_t tmem_d2 = tmem_d0 + (uint32_t)BT;
      if (a.splits == 1 && a.tma_epi != kEpiThreads) {
        // Staged epilogue.  Per chunk of tokens the warp reads its 32 rows in
        // the mma-fragment layout (16x256b: thread (g, t4) holds rows g, g + 8
        // of each 16-row half, token pairs 2 t4, +1), applies alpha / bias /
        // GELU and writes a [tokens][32 rows] box to shared memory, which lane 0
        // hands to TMA -- a store, or for the residual term (beta = 1) an
        // add-reduction performed at L2, so no old value is ever loaded.  f16:
        // 32-token chunks, f16 pairs along tokens packed and transposed by
        // stmatrix (256 outputs each), 64-byte rows with 64-byte swizzle
        // (16-byte chunk c of row k at c ^ ((k >> 1) & 3)); f32: 16-token
        // chunks, 128-byte rows, 128-byte swizzle.  Rows and tokens outside the
        // tensor are clipped by TMA.
        const int g = lane >> 2, t4 = lane & 3;
        const int nq = (tile % n_tiles) * 128 + q * 32;
        float bz[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int nn = nq + 8 * i + g;
          bz[i] = (a.bias && nn < a.N) ? __half2float(a.bias[nn]) : 0.0f;
        }
        uint8_t* ebuf = smem + L::kEOff + q * (2 * kEChunk);
        const bool gelu = (a.ydt & kOutGelu) != 0;
        const bool add = a.tma_epi == kEpiAdd;
        if (a.ydt & kOutF16) {
          // 32-token chunks, one 2 KB box per warp, rewritten once TMA has read
          // it (measured: the Efkolos prefill chain at M = 4096 took 2.35 ms with
          // two alternating 16-token boxes, 2.15 ms with this; 2.96 ms with
          // 8-token boxes): the per-chunk fence, warp sync and TMA issue dominate
#pragma unroll 1
          for (int c = 0; c < BT / 32 && m0 + c * 32 < a.M; c++) {
            uint32_t pk[2][2][4];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              uint32_t v[2][8];
              tc::tmem_ld_16x256b_x2(tmem_d + (uint32_t)(c * 32 + hh * 16), v[0]);
              tc::tmem_ld_16x256b_x2(tmem_d + (16u << 16) + (uint32_t)(c * 32 + hh * 16), v[1]);
              if (ISS == 2 && add2) {
                uint32_t u[2][8];
                tc::tmem_ld_16x256b_x2(tmem_d2 + (uint32_t)(c * 32 + hh * 16), u[0]);
                tc::tmem_ld_16x256b_x2(tmem_d2 + (16u << 16) + (uint32_t)(c * 32 + hh * 16), u[1]);
                tc::tmem_ld_wait_regs(u[0], u[1]);
                tc::reg_tie(v[0]);
                tc::reg_tie(v[1]);
                add_f32_regs(v[0], u[0]);
                add_f32_regs(v[1], u[1]);
              } else {
                tc::tmem_ld_wait();
              }
#pragma unroll
              for (int h = 0; h < 2; h++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                  // v[h][2e], v[h][2e+1]: row 16h + 8 (e & 1) + g of the warp,
                  // tokens 16 hh + 8 (e >> 1) + 2 t4, +1
                  const float b = bz[2 * h + (e & 1)];
                  float lo = fmaf(a.alpha, __uint_as_float(v[h][2 * e]), b);
                  float hi = fmaf(a.alpha, __uint_as_float(v[h][2 * e + 1]), b);
                  if (gelu) {
                    lo = gelu_fast(lo);
                    hi = gelu_fast(hi);
                  }
                  const __half2 p2 = __floats2half2_rn(lo, hi);
                  pk[hh][h][e] = *reinterpret_cast<const uint32_t*>(&p2);
                }
            }
            if (c >= 1) {
              if (lane == 0) tc::bulk_wait_read<0>();  // the previous box has been read
              __syncwarp();
            }
            // matrix mi = (rows 8 (mi & 1) .. +7 of half h, tokens 16 hh + 8 (mi >> 1) .. +7);
            // lane 8 mi + k addresses its column k
            const int mi = lane >> 3;
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              const int tk = hh * 16 + (lane & 7) + 8 * (mi >> 1);
#pragma unroll
              for (int h = 0; h < 2; h++) {
                const int chunk = 2 * h + (mi & 1);
                tc::stmatrix_x4_trans(tc::smem_u32(ebuf + tk * 64 + ((chunk ^ ((tk >> 1) & 3)) << 4)), pk[hh][h][0],
                                      pk[hh][h][1], pk[hh][h][2], pk[hh][h][3]);
              }
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (add)
                tc::tma_reduce_add_2d(&tmap_y, nq, m0 + c * 32, ebuf);
              else
                tc::tma_store_2d(&tmap_y, nq, m0 + c * 32, ebuf);
              tc::bulk_commit();
            }
          }
        } else {
          // f32: 16-token chunks, one 2 KB box [16 tokens][32 rows] (128-byte
          // rows, 128-byte swizzle: 16-byte chunk c of token row k at c ^ (k & 7));
          // each value is one 4-byte shared store, conflict-free (a warp's 32
          // stores cover 8 rows x 4 tokens in distinct banks)
#pragma unroll 1
          for (int c = 0; c < BT / 16 && m0 + c * 16 < a.M; c++) {
            if (c >= 1) {
              if (lane == 0) tc::bulk_wait_read<0>();
              __syncwarp();
            }
#pragma unroll 1
            for (int hh = 0; hh < 2; hh++) {  // two 8-token halves of the box
              uint32_t v[2][4];
              tc::tmem_ld_16x256b_x1(tmem_d + (uint32_t)(c * 16 + hh * 8), v[0]);
              tc::tmem_ld_16x256b_x1(tmem_d + (16u << 16) + (uint32_t)(c * 16 + hh * 8), v[1]);
              if (ISS == 2 && add2) {
                uint32_t u[2][4];
                tc::tmem_ld_16x256b_x1(tmem_d2 + (uint32_t)(c * 16 + hh * 8), u[0]);
                tc::tmem_ld_16x256b_x1(tmem_d2 + (16u << 16) + (uint32_t)(c * 16 + hh * 8), u[1]);
                tc::tmem_ld_wait_regs(u[0], u[1]);
                tc::reg_tie(v[0]);
                tc::reg_tie(v[1]);
                add_f32_regs(v[0], u[0]);
                add_f32_regs(v[1], u[1]);
              } else {
                tc::tmem_ld_wait();
              }
#pragma unroll
              for (int h = 0; h < 2; h++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                  // v[h][e]: row 16h + 8 (e >> 1) + g of the warp, token 8 hh + 2 t4 + (e & 1)
                  const int row = 16 * h + 8 * (e >> 1) + g, tk = 8 * hh + 2 * t4 + (e & 1);
                  float o = fmaf(a.alpha, __uint_as_float(v[h][e]), bz[2 * h + (e >> 1)]);
                  if (gelu) o = gelu_fast(o);
                  *reinterpret_cast<float*>(ebuf + tk * 128 + ((((row >> 2) ^ tk) & 7) << 4) + (row & 3) * 4) = o;
                }
            }
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (add)
                tc::tma_reduce_add_2d(&tmap_y, nq, m0 + c * 16, ebuf);
              else
                tc::tma_store_2d(&tmap_y, nq, m0 + c * 16, ebuf);
              tc::bulk_commit();
            }
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[buf]);
      } else if (a.splits == 1) {
#pragma unroll 1
        for (int cc = 0; cc < BT / 32; cc++) {
          uint32_t v[32];
          tc::tmem_ld_32x32b_x32(tmem_d + (uint32_t)(cc * 32), v);
          if (ISS == 2 && add2) {
            uint32_t u[32];
            tc::tmem_ld_32x32b_x32(tmem_d2 + (uint32_t)(cc * 32), u);
            tc::tmem_ld_wait();
            tc::reg_tie(u);
            tc::reg_tie(v);
            add_f32_regs(v, u);
          } else {
            tc::tmem_ld_wait();
          }
          const int tok0 = m0 + cc * 32;
          if (!row_ok || tok0 >= a.M) continue;
          const int ntok = min(32, a.M - tok0);
          float o[32];
#pragma unroll
          for (int jj = 0; jj < 32; jj++) o[jj] = fmaf(a.alpha, __uint_as_float(v[jj]), bias);
          store32(tok0, ntok, n, o);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[buf]);
      } else {
        // split-K: this unit's partial [BT tokens][128 rows] f32 to the workspace
        float* part = a.ws_part + (size_t)(tile * a.splits + split) * (128 * BT);
#pragma unroll 1
        for (int cc = 0; cc < BT / 32; cc++) {
          uint32_t v[32];
          tc::tmem_ld_32x32b_x32(tmem_d + (uint32_t)(cc * 32), v);
          if (ISS == 2 && add2) {
            uint32_t u[32];
            tc::tmem_ld_32x32b_x32(tmem_d2 + (uint32_t)(cc * 32), u);
            tc::tmem_ld_wait();
            tc::reg_tie(u);
            tc::reg_tie(v);
            add_f32_regs(v, u);
          } else {
            tc::tmem_ld_wait();
          }
#pragma unroll
          for (int jj = 0; jj < 32; jj++) part[(size_t)(cc * 32 + jj) * 128 + rr] = __uint_as_float(v[jj]);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[buf]);  // the accumulator is free again
        // publish, then count: the unit that completes a tile's quadrant adds the
        // tile's partials in slice order (no waiting on other CTAs)
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&a.ws_cnt[tile * 4 + q], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)(a.splits - 1)) {
          __threadfence();
          const float* p0 = a.ws_part + (size_t)tile * a.splits * (128 * BT) + rr;
          if (row_ok) {
            // 32 tokens at a time: every slice's partials of 8 tokens loaded before
            // the first add (up to 64 independent L2 loads in flight per lane)
            for (int t0 = 0; t0 < BT && m0 + t0 < a.M; t0 += 32) {
              float o[32];
#pragma unroll
              for (int h = 0; h < 4; h++) {
                float v[8][8];
#pragma unroll
                for (int sp = 0; sp < 8; sp++)
#pragma unroll
                  for (int u = 0; u < 8; u++)
                    v[sp][u] = sp < a.splits ? __ldcg(p0 + (size_t)sp * (128 * BT) + (size_t)(t0 + 8 * h + u) * 128)
                                             : 0.0f;
#pragma unroll
                for (int u = 0; u < 8; u++) {
                  float acc = 0.0f;
#pragma unroll
                  for (int sp = 0; sp < 8; sp++)
                    if (sp < a.splits) acc += v[sp][u];
                  o[8 * h + u] = fmaf(a.alpha, acc, bias);
                }
              }
              store32(m0 + t0, min(32, a.M - (m0 + t0)), n, o);
            }
          }
          __syncwarp();
          if (lane == 0) a.ws_cnt[tile * 4 + q] = 0u;  // leave the counter for the next call
        }
      }
    }
    // staged epilogue: the shared-memory boxes stay in use, and the outputs are
    // not final, until this thread's bulk groups complete
    if (lane == 0 && a.tma_epi != kEpiThreads) tc::bulk_wait_all();
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, kCols);
  }
}

// ------------------------------------------------------------------ host side

constexpr int kTcMaxDevices = 64;

// SM count of the current device (cached per device).
static int tc_num_sms() {
  static int sms[kTcMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kTcMaxDevices) {
    cudaGetLastError();
    return 148;
  }
  if (sms[dev] <= 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    sms[dev] = n;
  }
  return sms[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

template <int LAYOUT, int BT, int STAGES, int NACC, int ISS>
static cudaError_t launch_tc_t(const TcArgs& a, const __half* x, int ldx, cudaStream_t st, bool pdl) {
  using L = TcSmem<BT, STAGES>;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  const cuuint64_t gdim[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  const cuuint64_t gstride[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)BT};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // output boxes of the staged epilogue: [32 tokens][32 rows] f16 with 64-byte
  // swizzle or [16 tokens][32 rows] f32 with 128-byte swizzle (2 KB each)
  CUtensorMap tmy;
  memset(&tmy, 0, sizeof(tmy));
  if (a.tma_epi != kEpiThreads) {
    const cuuint64_t ydim[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    const bool f16 = (a.ydt & kOutF16) != 0;
    const cuuint64_t ystride[1] = {(cuuint64_t)a.ldy * (f16 ? 2 : 4)};
    const cuuint32_t ybox[2] = {32u, f16 ? 32u : 16u};
    r = enc(&tmy, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.y, ydim, ystride, ybox,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, f16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  auto kern = gemm_tc_kernel<LAYOUT, BT, STAGES, NACC, ISS>;
  // the shared-memory opt-in is a per-device property of the kernel: set it once
  // on every device this instance runs on (idempotent; a racing second set is harmless)
  static bool attr_set[kTcMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kTcMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int num_sms = tc_num_sms();
  const int n_tiles = (a.N + 127) / 128;
  const int num_tiles = n_tiles * ((a.M + BT - 1) / BT) * a.splits;  // work units
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_tiles < num_sms ? num_tiles : num_sms);
  cfg.blockDim = dim3(kTcThreads + 32 * (ISS - 1));
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, tm, tmy, a, n_tiles, num_tiles);
}

struct TcPlan {
  int bt = 64, nacc = 2, splits = 1;
  size_t ws_bytes = 0;  // workspace the plan needs (0 without split-K)
};

// Workspace layout: a fixed counter region first (one counter per tile and TMEM
// lane quadrant; at most kTcMaxSplitTiles tiles), then the f32 partials.  The
// counters sit at the same place for every shape and every call returns the
// ones it used to zero, so one workspace serves any sequence of shapes (the
// partials region is always written before it is read).
constexpr int kTcMaxSplitTiles = 1024;
constexpr size_t kTcCounterBytes = (size_t)kTcMaxSplitTiles * 4 * sizeof(unsigned);

static size_t tc_ws_bytes(int N, int M, int bt, int splits) {
  if (splits <= 1) return 0;
  const size_t tiles = (size_t)((N + 127) / 128) * ((M + bt - 1) / bt);
  return kTcCounterBytes + tiles * splits * 128 * bt * sizeof(float);
}

// Token-tile height BT and K split by a cost model: rounds of CTAs (work units
// / SMs, rounded up) x 128-k stages per unit x (fixed issue cost of a stage + 4
// cycles per token), plus, for a single accumulator, the exposed epilogue of
// every round after the first (epi_per_token cycles per token of the tile),
// plus, for a K split, each unit's partial write
// and the last unit's reduction (measured: 7-9 us per round at 64 tokens, fit
// as 10000 + 16 * S * BT in the same units).  The fixed ~640 cycles per stage
// is the MMA issuer's latency (two barrier waits, a fence, eight MMAs and two
// commits).  K splits are considered for 64- and 128-token tiles, with every
// slice at least two 128-k groups, when the workspace holds the plan's
// ws_bytes.  192-token tiles come with one accumulator (deeper A sub-rings; kept
// on ties, i.e. when the tiles fit one round) or two (the epilogue overlapped;
// measured on B200 at M = 4096: Efkolos LM head 255 -> 248 us, config-4
// ffn_down 508 -> 499 us, where the model picks it).
// cycles per token of a tile's epilogue, exposed after every round but the
// first when the tile has a single accumulator (measured with clock64 stamps in
// the MMA thread on B200: ~16k cycles per 256-token tile, with or without GELU;
// planning with it moved config-4 and Efkolos prefill shapes to double-buffered
// tiles: config-4 LM head at M = 4096 0.924 -> 0.732 ms, Efkolos prefill step
// 2.50 -> 2.35 ms)
constexpr int kTcEpiCyclesPerToken = 60;

static TcPlan plan_tc(int K, int N, int M, int sms, size_t ws_avail, int epi_per_token = kTcEpiCyclesPerToken) {
  struct Cand { int bt, nacc; };
  const Cand cands[] = {{64, 1}, {128, 2}, {192, 1}, {224, 1}, {256, 1}, {192, 2}};
  const int splits_c[] = {1, 2, 3, 4, 6, 8};  // the reduction unrolls up to 8 slices
  const long long n_tiles = (N + 127) / 128;
  const int KG = padded_k(K) / 128;
  const long long KT = KG;  // 128-k stages per tile
  TcPlan best;
  long long best_cost = -1;
  for (const Cand& c : cands) {
    if (c.bt > 64 && M <= 64) break;
    const long long tiles = n_tiles * ((M + c.bt - 1) / c.bt);
    for (int S : splits_c) {
      if (S > 1 && (c.bt > 128 || 2 * S > KG || tiles > kTcMaxSplitTiles)) continue;
      const size_t need = tc_ws_bytes(N, M, c.bt, S);
      if (S > 1 && need > ws_avail) continue;
      const long long units = tiles * S;
      const long long rounds = (units + sms - 1) / sms;
      const long long stages = (KT + S - 1) / S;
      long long cost = rounds * stages * (640 + 4 * c.bt);
      if (c.nacc == 1) cost += (rounds - 1) * (long long)epi_per_token * c.bt;
      if (S > 1) cost += rounds * (10000 + 16LL * S * c.bt);
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best.bt = c.bt;
        best.nacc = c.nacc;
        best.splits = S;
        best.ws_bytes = need;
      }
    }
  }
  return best;
}

size_t tc_workspace_bytes(int K, int N, int M) {
  return plan_tc(K, N, M, tc_num_sms(), (size_t)-1).ws_bytes;
}

// Workspace bytes the launcher's plan uses when ws_avail bytes are available
// (0: that plan does not split K).
size_t tc_workspace_used(int K, int N, int M, size_t ws_avail) {
  return plan_tc(K, N, M, tc_num_sms(), ws_avail).ws_bytes;
}

// Bytes at the start of a workspace that hold the split-K counters.
size_t tc_workspace_counter_bytes() { return kTcCounterBytes; }

// Tensor-core projection (prefill, and batched decode above 32 tokens).
// workspace: optional (nullptr / 0 bytes: no K split); its counter region must
// be zero before the first use and every call leaves it zero.
// wait_ns / no_x_loads: see TcArgs (the failure-path test hook passes a short
// limit and no X copies; every other caller the defaults).
cudaError_t launch_gemm_tc(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                           int ydt, int ldy, const __half* bias, float alpha, float beta, void* workspace,
                           size_t workspace_bytes, cudaStream_t st, bool pdl, bool const_weights,
                           unsigned long long wait_ns, bool no_x_loads) {
  TcArgs a;
  a.wait_ns = wait_ns;
  a.no_x_loads = no_x_loads ? 1 : 0;
  a.const_weights = const_weights ? 1 : 0;
  a.qs = tiled;
  a.scales = reinterpret_cast<const __half*>(tiled + tiled_scale_offset(K, N));
  a.K = K; a.N = N; a.Kp = padded_k(K); a.M = M;
  a.y = y; a.ydt = ydt; a.ldy = ldy; a.bias = bias; a.alpha = alpha; a.beta = beta;
  // outputs whose rows TMA can address (16-byte aligned base and row pitch)
  // take the staged epilogue when the residual term is absent or beta = 1
  const size_t esz = (ydt & kOutF16) ? 2 : 4;
  const bool tma_ok = ((uintptr_t)y & 15u) == 0 && ((size_t)ldy * esz) % 16 == 0;
  a.tma_epi = !tma_ok ? kEpiThreads : beta == 0.0f ? kEpiStore : beta == 1.0f ? kEpiAdd : kEpiThreads;
  const TcPlan p = plan_tc(K, N, M, tc_num_sms(), workspace ? workspace_bytes : 0);
  a.splits = p.splits;
  a.ws_part = nullptr;
  a.ws_cnt = nullptr;
  if (p.splits > 1) {
    a.ws_cnt = reinterpret_cast<unsigned*>(workspace);
    a.ws_part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kTcCounterBytes);
  }
  if (layout == 1) {
    switch (p.bt) {
      case 64: return launch_tc_t<1, 64, 6, 1, 2>(a, x, ldx, st, pdl);
      case 128: return launch_tc_t<1, 128, 3, 2, 1>(a, x, ldx, st, pdl);
      case 192: return p.nacc == 2 ? launch_tc_t<1, 192, 3, 2, 1>(a, x, ldx, st, pdl)
                                   : launch_tc_t<1, 192, 3, 1, 1>(a, x, ldx, st, pdl);
      case 224: return launch_tc_t<1, 224, 2, 1, 1>(a, x, ldx, st, pdl);
      default: return launch_tc_t<1, 256, 2, 1, 1>(a, x, ldx, st, pdl);
    }
  }
  switch (p.bt) {
    case 64: return launch_tc_t<0, 64, 6, 1, 2>(a, x, ldx, st, pdl);
    case 128: return launch_tc_t<0, 128, 3, 2, 1>(a, x, ldx, st, pdl);
    case 192: return p.nacc == 2 ? launch_tc_t<0, 192, 3, 2, 1>(a, x, ldx, st, pdl)
                                 : launch_tc_t<0, 192, 3, 1, 1>(a, x, ldx, st, pdl);
    case 224: return launch_tc_t<0, 224, 2, 1, 1>(a, x, ldx, st, pdl);
    default: return launch_tc_t<0, 256, 2, 1, 1>(a, x, ldx, st, pdl);
  }
}

// Reads and clears the device error flag (synchronous).
int take_device_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) cudaMemcpyToSymbol(tc::g_device_error, &zero, sizeof(int));
  return v;
}

}  // namespace aria_q4
