// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference counterpart: PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs (attn_fwd: one
// block per (query, head), fp32 SIMT).  One CTA owns two consecutive 128-query tiles (A and B) of
// one (batch, head) and streams the 128-key tiles they need once:
//
//   warp 8      TMA producer: Q_A and Q_B once, then K_j / V_j into a 3-stage ring
//   warp 9      MMA issuer (one thread), per key tile j, in this order:
//                 PV_A(j-1), S_A(j), PV_B(j-1), S_B(j)
//               S_w = Q_w K_j^T lands in TMEM (128 columns per tile); O_w += P_w V_j accumulates
//               in TMEM.  Because one commit covers every earlier MMA of the issuing thread, the
//               commit that announces S_w(j) also proves PV_w(j-1) finished: softmax warpgroup w
//               may then rewrite P_w and rescale O_w without another barrier.
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B (thread = query row = TMEM lane):
//               the whole 128-key row is read from TMEM at once, p = 2^(s*c - m*c) with
//               c = scale*log2(e) on the SFU, and bf16 P is written back to TMEM (two keys per
//               column), where the PV MMA reads its A operand; P never touches shared memory.
//               The running max is only moved (and O rescaled in TMEM) when a warp sees a row max
//               grow by more than 2^8, so most tiles skip the O round trip.  The two warpgroups alternate: one computes exponentials while the
//               tensor cores run the other's MMAs.
//   epilogue    O / l in bf16, lse = m*scale + ln(l) (the backward's convention)
//
// Heavy (late) tile pairs are scheduled first.  Every wait is bounded and unwinds on timeout.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pcb {
namespace fa {

constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kStages = 3;
constexpr int kThreads = 384;  // warpgroups 0, 1: softmax; warpgroup 2: TMA warp, MMA warp, two idle warps
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512); warpgroup 2 drops to
// 72 (frees 4 x 32 x 96 = 12288), the softmax warpgroups rise to 216 (take 2 x 4 x 32 x 48 = 12288).
constexpr int kRegsCtl = 72;
constexpr int kRegsSoftmax = 216;
static_assert(4 * 32 * (2 * kRegsSoftmax + kRegsCtl) <= kThreads * 168, "register split exceeds the launch");
constexpr int kAtom = 128 * 128;  // bytes of one [128 rows x 64 bf16] swizzled atom
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // move the running max only when it grows by more than 2^8

template <int HD>
struct Cfg {
  static constexpr int ATOMS = HD / 64;
  static constexpr int Q_OFF = 0;                                   // 2 buffers x tiles A, B
  static constexpr int K_OFF = Q_OFF + 2 * 2 * ATOMS * kAtom;       // kStages stages
  static constexpr int V_OFF = K_OFF + kStages * ATOMS * kAtom;     // kStages stages
  static constexpr int BAR_OFF = V_OFF + kStages * ATOMS * kAtom;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
  static constexpr int TM_S = 0;                                    // + w * 128
  static constexpr int TM_O = 2 * kBKV;                             // + w * HD
  static constexpr int TM_P = TM_O + 2 * HD;                        // + w * 64: bf16 P, two keys per column
  static_assert(TM_P + 2 * 64 <= 512, "TMEM budget");
};
static_assert(Cfg<64>::SMEM <= 232448, "shared memory budget");

// Work item i of the heavy-first list: tile pair t (query rows 256t..256t+255), batch-head bh.
struct Item {
  int t, b, h, bh;
};
PCB_DEVICE Item item_of(int i, int BH, int T, int H) {
  Item it;
  it.t = T - 1 - i / BH;
  it.bh = i % BH;
  it.b = it.bh / H;
  it.h = it.bh % H;
  return it;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, __nv_bfloat16* __restrict__ out, long long ld_o,
                       float* __restrict__ lse, int S, int H, int BH, float scale, int* err) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;                 // [2]
  uint64_t* q_empty = bars + 2;                // [2]
  uint64_t* kv_full = bars + 4;                // [kStages]
  uint64_t* kv_empty = kv_full + kStages;      // [kStages]
  uint64_t* s_full = kv_empty + kStages;       // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* o_final = p_full + 2;              // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = S / (2 * kBQ);
  const int n_items = T * BH;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) prefetch_tmap(&tm);
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= 8) {
    // control warpgroup: registers down, then the TMA warp and the MMA warp
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
    if (warp == 8 && lane == 0) {
      // ---------------- TMA producer: runs ahead into the next item ----------------
      int qc = 0, kc = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++qc) {
        const Item it = item_of(i, BH, T, H);
        const int qb = qc & 1;
        if (!(ok = mbar_wait(&q_empty[qb], ((qc >> 1) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
        mbar_arrive_expect_tx(&q_full[qb], 2 * C::ATOMS * kAtom);
        const int row0 = it.b * S + it.t * 2 * kBQ;
#pragma unroll
        for (int w = 0; w < 2; ++w)
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_2d(sQ + ((qb * 2 + w) * C::ATOMS + a) * kAtom, &tm, &q_full[qb], it.h * HD + a * 64,
                        row0 + w * kBQ);
        const int n_kv = 2 * it.t + 2;
        for (int j = 0; j < n_kv; ++j, ++kc) {
          const int st = kc % kStages;
          if (!(ok = mbar_wait(&kv_empty[st], ((kc / kStages) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
          mbar_arrive_expect_tx(&kv_full[st], 2 * C::ATOMS * kAtom);
          const int krow = it.b * S + j * kBKV;
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a) {
            tma_load_2d(sK + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (H + it.h) * HD + a * 64, krow);
            tma_load_2d(sV + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (2 * H + it.h) * HD + a * 64, krow);
          }
        }
      }
    } else if (warp == 9 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16(kBQ, kBKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBQ, HD, 0, 1);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto kv_ready = [&](int n) -> bool {
        return mbar_wait(&kv_full[n % kStages], (n / kStages) & 1, err, kErrTimeoutFull, abort_flag);
      };
      auto issue_s = [&](int w, int qb, int n) {
        const uint32_t kb = k_addr + (n % kStages) * C::ATOMS * kAtom;
        const uint32_t qa = q_addr + (qb * 2 + w) * C::ATOMS * kAtom;
        const uint64_t ad = make_smem_desc(qa, 16, 1024, 2), bd = make_smem_desc(kb, 16, 1024, 2);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {  // advancing the start address = adding (bytes >> 4) to the descriptor
          const uint64_t off = ((k >> 2) * kAtom + (k & 3) * 32) >> 4;
          umma_bf16(tmem + C::TM_S + w * kBKV, ad + off, bd + off, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
      };
      auto issue_pv = [&](int w, int n, bool first) {  // A = P from TMEM (16 keys = 8 columns per step)
        const uint32_t vb = v_addr + (n % kStages) * C::ATOMS * kAtom;
        const uint64_t bd = make_smem_desc(vb, kAtom, 1024, 2);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBKV / 16; ++k)
          umma_bf16_ts(tmem + C::TM_O + w * HD, tmem + C::TM_P + w * 64 + k * 8, bd + (k * 2048 >> 4), idesc_o,
                       (!first || k > 0) ? 1u : 0u);
      };
      int qc = 0, kc = 0, ta = 0, tb = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++qc) {
        const Item it = item_of(i, BH, T, H);
        const int qb = qc & 1;
        const int last_a = 2 * it.t, n_kv = 2 * it.t + 2;
        // S_w(0) may overwrite S_w: the previous item's last p_full_w (waited below) proved it was read
        if (!(ok = mbar_wait(&q_full[qb], (qc >> 1) & 1, err, kErrTimeoutFull, abort_flag) && kv_ready(kc))) break;
        issue_s(0, qb, kc);
        issue_s(1, qb, kc);
        for (int j = 0; j < n_kv; ++j) {
          const int n = kc + j;
          if (j <= last_a) {
            if (!(ok = mbar_wait(&p_full[0], ta & 1, err, kErrTimeoutTmemEmpty, abort_flag))) break;
            ++ta;
            issue_pv(0, n, j == 0);
            if (j + 1 <= last_a) {
              if (!(ok = kv_ready(n + 1))) break;
              issue_s(0, qb, n + 1);
            } else {
              umma_commit(&o_final[0]);
            }
          }
          if (!(ok = mbar_wait(&p_full[1], tb & 1, err, kErrTimeoutTmemEmpty, abort_flag))) break;
          ++tb;
          issue_pv(1, n, j == 0);
          umma_commit(&kv_empty[n % kStages]);
          if (j + 1 < n_kv) {
            if (!(ok = kv_ready(n + 1))) break;
            issue_s(1, qb, n + 1);
          } else {
            umma_commit(&q_empty[qb]);
            umma_commit(&o_final[1]);
          }
        }
        kc += n_kv;
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ---------------- softmax warpgroups: one query row per thread ----------------
    const int w = warp >> 2;                    // 0 = tile A, 1 = tile B
    const int r = threadIdx.x & 127;            // row within the tile == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = lane_base + C::TM_S + w * kBKV;
    const uint32_t o_col = lane_base + C::TM_O + w * HD;
    const uint32_t p_col = lane_base + C::TM_P + w * 64;
    const float c = scale * kLog2e;
    int tc = 0, ic = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++ic) {
      const Item it = item_of(i, BH, T, H);
      const int last = 2 * it.t + w;           // tile A: key tiles 0..2t, tile B: 0..2t+1
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j <= last; ++j, ++tc) {
        ok = mbar_wait(&s_full[w], tc & 1, err, kErrTimeoutTmemFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        uint32_t sv_u[128];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          tmem_ld_32x32b_x32(s_col + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(sv_u + cc * 32));
        tmem_ld_wait();
#define SV(e) __uint_as_float(sv_u[e])
        if (j == last) {  // diagonal tile: key column e is visible to row r iff e <= r
#pragma unroll
          for (int e = 0; e < 128; ++e) sv_u[e] = e <= r ? sv_u[e] : __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = SV(e);
#pragma unroll
        for (int e = 8; e < 128; ++e) mx[e & 7] = fmaxf(mx[e & 7], SV(e));
        const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        const float m_new = fmaxf(m, tmax);
        const bool grow = (m_new - m) * c > kRescaleLog2;  // always true on the first tile (m = -inf)
        const bool rescale = __any_sync(0xffffffffu, grow);
        float corr = 1.f;
        if (rescale) {
          corr = ex2_approx((m - m_new) * c);  // 0 when m = -inf
          m = m_new;
          l *= corr;
        }
        const float msc = m * c;
        float rsv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {  // keys 32*q4 .. 32*q4+31 -> 16 TMEM columns of bf16 pairs
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = ex2_approx(fmaf(SV(q4 * 32 + e), c, -msc));
            const float p1 = ex2_approx(fmaf(SV(q4 * 32 + e + 1), c, -msc));
            rsv[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_bf16x2(p0, p1);
          }
          tmem_st_32x32b_x16(p_col + q4 * 16, pk);
        }
#undef SV
        l += (rsv[0] + rsv[1]) + (rsv[2] + rsv[3]);
        if (rescale && j > 0) {  // O holds PV(0..j-1): scale it in place (PV_w(j-1) is complete, see above)
#pragma unroll 1
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(o_col + cc * 32, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * corr);
            tmem_st_32x32b_x32(o_col + cc * 32, ov);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[w]);
      }
      if (!ok) break;
      ok = mbar_wait(&o_final[w], ic & 1, err, kErrTimeoutTmemFull, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      // epilogue: the next item's PV_w(0) overwrites O_w only after this warpgroup's next p_full_w,
      // which it signals after these loads completed
      const int q = it.t * 2 * kBQ + w * kBQ + r;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (long long)(it.b * S + q) * ld_o + it.h * HD;
#pragma unroll
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_col + cc * 32, ov);
        tmem_ld_wait();
#pragma unroll
        for (int d = 0; d < 32; d += 8) {
          uint4 v = make_uint4(
              pack_bf16x2(__uint_as_float(ov[d]) * inv, __uint_as_float(ov[d + 1]) * inv),
              pack_bf16x2(__uint_as_float(ov[d + 2]) * inv, __uint_as_float(ov[d + 3]) * inv),
              pack_bf16x2(__uint_as_float(ov[d + 4]) * inv, __uint_as_float(ov[d + 5]) * inv),
              pack_bf16x2(__uint_as_float(ov[d + 6]) * inv, __uint_as_float(ov[d + 7]) * inv));
          *reinterpret_cast<uint4*>(orow + cc * 32 + d) = v;
        }
      }
      lse[(long long)it.bh * S + q] = m * scale + logf(l);
      tc_fence_before();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

}  // namespace fa

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_fa() {
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

template <int HD>
static int fa_launch(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                     float scale, int* err, cudaStream_t s) {
  using C = fa::Cfg<HD>;
  auto fn = encode_fn_fa();
  if (!fn) return -5;
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(3 * H * HD), static_cast<cuuint64_t>(B) * S};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  if (fn(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -5;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fa::attn_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    attr = true;
  }
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_sms <= 0) num_sms = 148;
  }
  const int n_items = B * H * (S / (2 * fa::kBQ));
  const int grid = n_items < num_sms ? n_items : num_sms;  // persistent: one CTA per SM
  fa::attn_fwd_tc_kernel<HD><<<grid, fa::kThreads, C::SMEM, s>>>(tm, reinterpret_cast<__nv_bfloat16*>(out), ld_o,
                                                                   lse, S, H, B * H, scale, err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(1000 + static_cast<int>(e));
}

}  // namespace pcb

// Same contract as pcb_attn_fwd (qkv [B*S, 3*H*HD] bf16 with q|k|v column blocks, out [B*S, H*HD]
// bf16, lse [B*H, S] fp32), on tcgen05.  S % 256 == 0, HD == 64, row strides % 8 == 0.
int pcb_attn_fwd_tc(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                    int HD, float scale, int* err, cudaStream_t s) {
  if (S % 256 != 0 || ld % 8 || ld_o % 8) return -1;
  if (reinterpret_cast<uintptr_t>(qkv) & 15) return -1;
  if (HD == 64) return pcb::fa_launch<64>(qkv, ld, out, ld_o, lse, B, S, H, scale, err, s);
  return -1;
}
