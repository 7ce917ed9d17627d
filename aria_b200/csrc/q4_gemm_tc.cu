// q4_gemm_tc.cu -- prefill-regime Q4_0 projection on the 5th-generation tensor
// cores (tcgen05, sm_100a).
//
// Replaces, for Q4_0 weights and M > 32 tokens, the cuBLAS fp16 GEMM of
// lold3344/ARIA's forward pass (`gemm()` src/transformer_cuda.rs:615-640 at
// :1583, :1686, :1753, :1805, :1864), which there runs with M = t tokens
// (forward_gpu recomputes the whole prompt every step).
//
// One CTA computes D[128 weight rows][BT tokens] = W_tile[128 x K] . X_tile[BT x K]^T
// ("swap AB": the weights are the 128-row UMMA operand, so each dequantised weight
// serves BT = up to 256 tokens):
//   warp 4      TMA producer: X tiles [BT x 64 k] f16, 128-byte swizzle, no multicast
//   warps 0-3   dequantisers: one weight row per thread; the row's 128-k group of
//               codes (64 B) is read straight from global memory into registers,
//               turned into (q-8)*scale f16 (LOP3/HSUB/HMUL), and written as 16-byte
//               chunks into the 128-byte-swizzled K-major A tile; then the epilogue
//   warp 5      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BT, K=16,
//               f16 x f16 -> f32 accumulator in TMEM), tcgen05.commit to release stages
// Stages are mbarrier-ring buffered (STAGES deep).  Every wait is bounded (one
// second); on expiry the kernel records an error code in g_device_error, unwinds,
// frees its TMEM and returns instead of hanging the GPU.
//
// The dequantised weight is rounded once to f16 ((q-8)*scale, relative error
// <= 2^-11 per weight); products and sums are f32 in the tensor core.
#include <cuda.h>

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
};

constexpr int kTcThreads = 192;
constexpr int kBK = 64;                   // k per pipeline stage (one 128-byte swizzle row of f16)
constexpr int kATileBytes = 128 * kBK * 2;  // 16 KB

template <int BT, int STAGES>
struct TcSmem {
  static constexpr int kXTile = BT * kBK * 2;
  static constexpr int kStage = kXTile + kATileBytes;
  static constexpr int kBarOff = STAGES * kStage;
  static constexpr int kBytes = kBarOff + 256 + 1024;  // barriers + alignment slack
};

template <int LAYOUT, int BT, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const TcArgs a) {
  using L = TcSmem<BT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_x = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full_a = full_x + STAGES;
  uint64_t* empty = full_a + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128;
  const int m0 = blockIdx.y * BT;
  const int KT = (a.K + kBK - 1) / kBK;
  constexpr uint32_t kCols = BT < 32 ? 32 : BT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full_x[s], 1);
      tc::mbar_init(&full_a[s], 128);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accum, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(tmem_slot, kCols);
    tc::tmem_relinquish();
  }
  if (warp == 4 && lane == 0) tc::prefetch_tmap(&tmap_x);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  grid_dep_launch();
  grid_dep_wait();

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < KT; it++) {
        const int s = it % STAGES;
        if (it >= STAGES && !tc::mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) {
          tc::record_error(tc::kErrTimeoutEmpty);
          break;
        }
        uint8_t* xs = smem + s * L::kStage;
        tc::mbar_arrive_expect_tx(&full_x[s], L::kXTile);
        tc::tma_load_2d(xs, &tmap_x, it * kBK, m0, &full_x[s]);
        issued = it + 1;
      }
      // drain: never leave the CTA while a copy into its shared memory is in flight
      for (int it = (issued > STAGES ? issued - STAGES : 0); it < issued; it++)
        tc::mbar_wait(&full_x[it % STAGES], (it / STAGES) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16_f32(128, BT);
      bool ok = true;
      for (int it = 0; it < KT && ok; it++) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!tc::mbar_wait(&full_x[s], ph) || !tc::mbar_wait(&full_a[s], ph)) {
          tc::record_error(tc::kErrTimeoutFull);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t xs = tc::smem_u32(smem + s * L::kStage);
        const uint32_t as = xs + L::kXTile;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++) {
          const uint64_t adesc = tc::sdesc_k_sw128(as + kk * 32);
          const uint64_t bdesc = tc::sdesc_k_sw128(xs + kk * 32);
          tc::umma_f16(tmem_d, adesc, bdesc, idesc, (it > 0 || kk > 0) ? 1u : 0u);
        }
        tc::umma_commit(&empty[s]);
      }
      if (!ok) atomicExch(abort_flag, 1);
      tc::umma_commit(accum);
    }
  } else {
    // ------------------------------------------------------------ dequantisers
    const int r = threadIdx.x;  // 0..127: weight row n0 + r
    const int n = n0 + r;
    const bool row_ok = n < a.N;
    const size_t RB = (size_t)a.Kp >> 1;
    const uint8_t* qrow = a.qs + (size_t)n * RB;
    const int KB = a.Kp >> 5;
    const int grp = n >> 5;
    uint4 gq[4], gq_next[4];
    uint2 gs = make_uint2(0, 0), gs_next = make_uint2(0, 0);
    auto load_group = [&](int G, uint4 (&q)[4], uint2& sc) {
      if (row_ok && G * 128 < a.Kp) {
#pragma unroll
        for (int j = 0; j < 4; j++) q[j] = ld_stream_u4(qrow + (size_t)G * 64 + 16 * j);
        if (LAYOUT == 1) sc = __ldg(reinterpret_cast<const uint2*>(a.scales + (size_t)n * KB + 4 * G));
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) q[j] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        sc = make_uint2(0, 0);
      }
    };
    load_group(0, gq_next, gs_next);
    bool ok = true;
    for (int it = 0; it < KT; it++) {
      const int s = it % STAGES;
      const int G = it >> 1, h = it & 1;
      if (h == 0) {
#pragma unroll
        for (int j = 0; j < 4; j++) gq[j] = gq_next[j];
        gs = gs_next;
        load_group(G + 1, gq_next, gs_next);  // one group ahead
      }
      if (it >= STAGES && !tc::mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) {
        tc::record_error(tc::kErrTimeoutEmpty);
        ok = false;
        break;
      }
      uint8_t* arow = smem + s * L::kStage + L::kXTile + r * 128;
      // words (t, i) with i in {2h, 2h+1}: local k = 32*(i-2h) + 8t, chunk c = 4*(i-2h) + t
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const uint4 q = gq[t];
#pragma unroll
        for (int ii = 0; ii < 2; ii++) {
          const int i = 2 * h + ii;
          const uint32_t w = (i == 0) ? q.x : (i == 1) ? q.y : (i == 2) ? q.z : q.w;
          uint32_t d[4];
          dequant_word_f16x2(w, d);
          if (LAYOUT == 1) {
            const uint32_t sw = (i < 2) ? gs.x : gs.y;
            const uint32_t s1 = (i & 1) ? (sw >> 16) : (sw & 0xFFFFu);
            const uint32_t s2 = s1 | (s1 << 16);
#pragma unroll
            for (int e = 0; e < 4; e++) d[e] = hmul2_u32(d[e], s2);
          } else {
            const int kk = G * 128 + 32 * i + 8 * t;
            const uint4 s8 = row_ok ? __ldg(reinterpret_cast<const uint4*>(a.scales + (size_t)grp * a.Kp + kk))
                                    : make_uint4(0, 0, 0, 0);
            d[0] = hmul2_u32(d[0], s8.x);
            d[1] = hmul2_u32(d[1], s8.y);
            d[2] = hmul2_u32(d[2], s8.z);
            d[3] = hmul2_u32(d[3], s8.w);
          }
          const int c = 4 * ii + t;
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) = make_uint4(d[0], d[1], d[2], d[3]);
        }
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&full_a[s]);
    }
    if (!ok) atomicExch(abort_flag, 1);

    // ------------------------------------------------------------ epilogue
    if (!tc::mbar_wait(accum, 0)) {
      tc::record_error(tc::kErrTimeoutAccum);
    } else if (*reinterpret_cast<volatile int*>(abort_flag) == 0) {
      tc::tc_fence_after();
      const float bias = (a.bias && row_ok) ? __half2float(a.bias[n]) : 0.0f;
#pragma unroll 1
      for (int cc = 0; cc < BT / 32; cc++) {
        uint32_t v[32];
        tc::tmem_ld_32x32b_x32(tmem_d + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cc * 32), v);
        tc::tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int tok = m0 + cc * 32 + j;
            if (tok < a.M) {
              float o = a.alpha * __uint_as_float(v[j]) + bias;
              const size_t idx = (size_t)tok * a.ldy + n;
              if (a.ydt == 0) {
                float* yp = reinterpret_cast<float*>(a.y) + idx;
                if (a.beta != 0.0f) o += a.beta * *yp;
                *yp = o;
              } else {
                __half* yp = reinterpret_cast<__half*>(a.y) + idx;
                if (a.beta != 0.0f) o += a.beta * __half2float(*yp);
                *yp = __float2half_rn(o);
              }
            }
          }
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_d, kCols);
  }
}

// ------------------------------------------------------------------ host side

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

template <int LAYOUT, int BT, int STAGES>
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
  auto kern = gemm_tc_kernel<LAYOUT, BT, STAGES>;
  static bool attr_set = false;  // idempotent; a racing second set is harmless
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + 127) / 128, (a.M + BT - 1) / BT);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, tm, a);
}

// Prefill-regime projection (M > 32).  BT (tokens per CTA) follows M.
cudaError_t launch_gemm_tc(const uint8_t* tiled, int layout, int K, int N, const __half* x, int M, int ldx, void* y,
                           int ydt, int ldy, const __half* bias, float alpha, float beta, cudaStream_t st, bool pdl) {
  TcArgs a;
  a.qs = tiled;
  a.scales = reinterpret_cast<const __half*>(tiled + tiled_scale_offset(K, N));
  a.K = K; a.N = N; a.Kp = padded_k(K); a.M = M;
  a.y = y; a.ydt = ydt; a.ldy = ldy; a.bias = bias; a.alpha = alpha; a.beta = beta;
  if (layout == 1) {
    if (M <= 32) return launch_tc_t<1, 32, 8>(a, x, ldx, st, pdl);
    if (M <= 64) return launch_tc_t<1, 64, 8>(a, x, ldx, st, pdl);
    if (M <= 128) return launch_tc_t<1, 128, 6>(a, x, ldx, st, pdl);
    return launch_tc_t<1, 256, 4>(a, x, ldx, st, pdl);
  }
  if (M <= 32) return launch_tc_t<0, 32, 8>(a, x, ldx, st, pdl);
  if (M <= 64) return launch_tc_t<0, 64, 8>(a, x, ldx, st, pdl);
  if (M <= 128) return launch_tc_t<0, 128, 6>(a, x, ldx, st, pdl);
  return launch_tc_t<0, 256, 4>(a, x, ldx, st, pdl);
}

// Reads and clears the device error flag (synchronous).
int take_device_error() {
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) cudaMemcpyToSymbol(tc::g_device_error, &zero, sizeof(int));
  return v;
}

}  // namespace aria_q4
