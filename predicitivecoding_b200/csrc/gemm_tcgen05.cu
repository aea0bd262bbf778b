// tcgen05 GEMM kernel + host launcher.  See gemm_tcgen05.cuh for the design.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm_epilogue.cuh"

namespace pcb {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;                 // two per TMEM lane quadrant, splitting columns
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer warp + MMA warp + epilogue warps

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (args.M + kBM - 1) / kBM;
  const int num_n = (args.N + BN - 1) / BN;
  const int total_kb = (args.K + kBK - 1) / kBK;
  const int tiles = num_m * num_n * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int split = tile % args.splits;
        const int rest = tile / args.splits;
        const int mb = rest % num_m, nb = rest / num_m;
        const int m0 = mb * kBM, n0 = nb * BN;
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(total_kb, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrTimeoutEmpty, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const int k0 = kb * kBK;
          if (args.a_mn == 0) {
            tma_load_2d(sa, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int p = 0; p < kBM / 64; ++p) tma_load_2d(sa + p * 8192, &tmA, &full[stage], m0 + 64 * p, k0);
          }
          if (args.b_mn == 0) {
            tma_load_2d(sb, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int p = 0; p < BN / 64; ++p) tma_load_2d(sb + p * 8192, &tmB, &full[stage], n0 + 64 * p, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // let copies already in flight land before the CTA's smem goes away
        for (int s = 0; s < STAGES; ++s) {
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_u32(&full[s]), 0) && !mbar_try_wait(smem_u32(&full[s]), 1) &&
                 clock64() - t0 < 1000000LL) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = make_idesc_bf16(kBM, BN, args.a_mn, args.b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int split = tile % args.splits;
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(total_kb, kb0 + args.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.err, kErrTimeoutTmemEmpty, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = args.a_mn ? make_smem_desc(sa + k * 2048, 8192, 1024, 2)
                                          : make_smem_desc(sa + k * 32, 16, 1024, 2);
            const uint64_t bd = args.b_mn ? make_smem_desc(sb + k * 2048, 8192, 1024, 2)
                                          : make_smem_desc(sb + k * 32, 16, 1024, 2);
            umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;             // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;   // which of the two warps of this quadrant (column split)
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int rest = tile / args.splits;
      const int mb = rest % num_m, nb = rest / num_m;
      const int m = mb * kBM + row;
      const int n0 = nb * BN;
      const bool row_ok = m < args.M;
      if (!mbar_wait(&tfull[acc], acc_phase, args.err, kErrTimeoutTmemFull, abort_flag)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (EPI == EPI_SWIGLU) {
        // 128-column groups: [64 gate | 64 up]; output 64 activation columns per group
#pragma unroll 1
        for (int g = 0; g < BN / 128; ++g) {
          {
            const int h = half;
            float gv[32], uv[32];
            tmem_load_f32x32(tbase + g * 128 + h * 32, gv);
            tmem_load_f32x32(tbase + g * 128 + 64 + h * 32, uv);
            const int ncol = n0 + g * 128 + h * 32;  // gate column in pre
            const int nvalid = min(32, args.N - ncol);
            if (row_ok && nvalid > 0) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                gv[j] *= args.alpha;
                uv[j] *= args.alpha;
              }
              __nv_bfloat16* pre = reinterpret_cast<__nv_bfloat16*>(args.C) + (long long)m * args.ldc;
              store_bf16x32(pre + ncol, gv, nvalid);
              store_bf16x32(pre + ncol + 64, uv, nvalid);
              float o[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                // activation uses the bf16-rounded pre values so that the backward
                // (which reads them back) sees exactly what the forward used
                const float gg = __bfloat162float(__float2bfloat16_rn(gv[j]));
                const float uu = __bfloat162float(__float2bfloat16_rn(uv[j]));
                o[j] = __fdividef(gg, 1.f + __expf(-gg)) * uu;
              }
              const int fcol = (n0 >> 1) + g * 64 + h * 32;
              store_bf16x32(reinterpret_cast<__nv_bfloat16*>(args.D) + (long long)m * args.ldd + fcol, o, nvalid);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          tmem_load_f32x32(tbase + c * 32, v);
          epilogue_chunk<EPI>(args, m, n0 + c * 32, v, row_ok);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 2-D map with 128-byte swizzle; box inner extent must be 64 elements.
static bool make_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                     uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int EPI>
static int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t s) {
  using Cfg = GemmCfg<BN>;
  static bool attr_done = false;  // per instantiation; set once (thread-safe enough: idempotent)
  if (!attr_done) {
    cudaFuncSetAttribute(gemm_tcgen05_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    attr_done = true;
  }
  gemm_tcgen05_kernel<BN, EPI><<<grid, kThreads, Cfg::SMEM_BYTES, s>>>(ta, tb, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int BN>
static int dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                        cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_one<BN, EPI_BF16>(ta, tb, a, grid, s);
    case EPI_F32: return launch_one<BN, EPI_F32>(ta, tb, a, grid, s);
    case EPI_ACC_F32: return launch_one<BN, EPI_ACC_F32>(ta, tb, a, grid, s);
    case EPI_RED_F32: return launch_one<BN, EPI_RED_F32>(ta, tb, a, grid, s);
    case EPI_GELU: return launch_one<BN, EPI_GELU>(ta, tb, a, grid, s);
    case EPI_SWIGLU: return launch_one<BN, EPI_SWIGLU>(ta, tb, a, grid, s);
    case EPI_SWIGLU_BWD: return launch_one<BN, EPI_SWIGLU_BWD>(ta, tb, a, grid, s);
    case EPI_GELU_BWD: return launch_one<BN, EPI_GELU_BWD>(ta, tb, a, grid, s);
    case EPI_PC_PRED: return launch_one<BN, EPI_PC_PRED>(ta, tb, a, grid, s);
    case EPI_PC_STATE: return launch_one<BN, EPI_PC_STATE>(ta, tb, a, grid, s);
    case EPI_PC_WUPD: return launch_one<BN, EPI_PC_WUPD>(ta, tb, a, grid, s);
    case EPI_BF16_ACC: return launch_one<BN, EPI_BF16_ACC>(ta, tb, a, grid, s);
    case EPI_RESID_F32: return launch_one<BN, EPI_RESID_F32>(ta, tb, a, grid, s);
    case EPI_RS_BF16: return launch_one<BN, EPI_RS_BF16>(ta, tb, a, grid, s);
    default: return -2;
  }
}

}  // namespace pcb

using namespace pcb;

int pcb_gemm_pair_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, int epi,
                         GemmArgs args, int bn, int splits, int num_sms, cudaStream_t stream);

// 0 = choose per problem, 1 = single-CTA kernel only, 2 = CTA-pair kernel whenever legal.
// Read once from PCB_GEMM_MODE ("auto" | "single" | "pair").
static int g_gemm_mode_override = -1;
extern "C" void pcb_set_gemm_mode(int mode) { g_gemm_mode_override = mode; }
static int gemm_mode() {
  if (g_gemm_mode_override >= 0) return g_gemm_mode_override;
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PCB_GEMM_MODE");
    mode = 0;
    if (e && strcmp(e, "single") == 0) mode = 1;
    if (e && strcmp(e, "pair") == 0) mode = 2;
  }
  return mode;
}

// Split-K count for the atomic (EPI_RED_F32) epilogue: the split s minimising
//   waves(s) * (k-blocks per split + per-tile overhead),  waves(s) = ceil(tiles * s / slots),
// i.e. the one that fills the persistent grid best without paying more tile prologues/epilogues
// than the extra parallelism buys.  The overhead is counted as 8 k-blocks per tile.
static int pick_splits(int tiles, int total_kb, int slots) {
  int best = 1;
  long long best_cost = -1;
  for (int sp = 1; sp <= 16; ++sp) {
    if (sp > 1 && total_kb / sp < 4) break;
    const long long waves = ((long long)tiles * sp + slots - 1) / slots;
    const long long cost = waves * ((total_kb + sp - 1) / sp + 8);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

int pcb_gemm_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, int epi,
                    GemmArgs args, int force_bn, int force_splits, int num_sms, cudaStream_t stream) {
  const int M = args.M, N = args.N, K = args.K;
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  // TMA: global strides must be multiples of 16 bytes, base 16-byte aligned.
  if ((lda % 8) != 0 || (ldb % 8) != 0) return -1;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) return -1;
  if (epi < 0 || epi >= EPI_COUNT) return -2;
  if (num_sms <= 0) num_sms = 148;
  args.a_mn = a_mn;
  args.b_mn = b_mn;

  const int num_m = (M + kBM - 1) / kBM;
  const int total_kb = (K + kBK - 1) / kBK;
  if (args.ag_world > 1) {  // fused all-gather exists only in the CTA-pair kernel
    const int pbn = (force_bn == 128 || force_bn == 256) ? force_bn : (N >= 256 ? 256 : 128);
    return pcb_gemm_pair_launch(A, a_mn, lda, B, b_mn, ldb, epi, args, pbn, 1, num_sms, stream);
  }
  {
    // CTA pairs (256-row tiles, half the B traffic per SM) when the problem has enough pair tiles
    const int mode = gemm_mode();
    const int pbn = (force_bn == 128 || force_bn == 256) ? force_bn : (N >= 256 ? 256 : 128);
    const int ptiles = ((M + 255) / 256) * ((N + pbn - 1) / pbn);
    int psplits = force_splits > 0 ? force_splits : 1;
    if (force_splits <= 0 && epi == EPI_RED_F32) psplits = pick_splits(ptiles, total_kb, num_sms / 2);
    const bool legal = M >= 256 && (epi != EPI_SWIGLU || pbn % 128 == 0);
    const bool worth = ptiles * psplits >= num_sms / 4 && total_kb >= 4;
    if (mode != 1 && legal && (mode == 2 || worth))
      return pcb_gemm_pair_launch(A, a_mn, lda, B, b_mn, ldb, epi, args, pbn, psplits, num_sms, stream);
  }
  int bn = force_bn;
  if (bn != 128 && bn != 256) {
    const int tiles256 = num_m * ((N + 255) / 256);
    bn = (N >= 256 && tiles256 >= num_sms) ? 256 : 128;
  }
  const int num_n = (N + bn - 1) / bn;
  int splits = force_splits;
  if (splits <= 0) {
    splits = 1;
    if (epi == EPI_RED_F32) splits = pick_splits(num_m * num_n, total_kb, num_sms);
  }
  if (splits > 1 && epi != EPI_RED_F32) return -4;  // only the atomic epilogue may split K
  int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;  // every split has >= 1 k-block
  args.splits = splits;
  args.kb_per_split = kbps;

  CUtensorMap ta, tb;
  bool ok;
  if (a_mn == 0) ok = make_map(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, kBM);
  else ok = make_map(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 64);
  if (!ok) return -5;
  if (b_mn == 0) ok = make_map(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64, (uint32_t)bn);
  else ok = make_map(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, 64);
  if (!ok) return -5;

  const int tiles = num_m * num_n * splits;
  const int grid = tiles < num_sms ? tiles : num_sms;
  return bn == 256 ? dispatch_epi<256>(epi, ta, tb, args, grid, stream)
                   : dispatch_epi<128>(epi, ta, tb, args, grid, stream);
}
