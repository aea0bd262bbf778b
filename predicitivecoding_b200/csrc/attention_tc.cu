// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference counterpart: PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs (attn_fwd: one
// block per (query, head), fp32 SIMT).  One CTA owns two consecutive 128-query tiles (A and B) of
// one (batch, head) and streams the 128-key tiles they need once:
//
//   warp 8      TMA producer: Q_A and Q_B, then K_j / V_j into a ring
//   warp 9      MMA issuer (one thread): S_w = Q_w K_j^T into TMEM (128 columns per tile) and
//               O_w += P_w V_j accumulating in TMEM
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B (thread = query row = TMEM lane):
//               the whole 128-key row is read from TMEM at once, p = 2^(s*c - m*c) with
//               c = scale*log2(e) on the SFU, and bf16 P is written back to TMEM (two keys per
//               column), where the PV MMA reads its A operand; P never touches shared memory.
//               The running max is only moved (and O rescaled in TMEM) when a warp sees a row max
//               grow by more than 2^8, so most tiles skip the O round trip.
//   epilogue    O / l in bf16, lse = m*scale + ln(l) (the backward's convention)
//
// Head dim 64 (TMEM: S 2x128 + O 2x64 + P 2x64 = 512 columns): S and P live in separate columns,
// so a softmax warpgroup releases S (s_free) as soon as the row is in registers and the MMA issuer
// starts S_w(j+1) while the exponentials of tile j run; P_w(j+1) is stored only after the MMA that
// read P_w(j) has completed (pv_done).  Issue order per key tile: S_A(j+1), S_B(j+1), PV_A(j),
// PV_B(j).
// Head dim 128 (TMEM: S 2x128 + O 2x128): P is written over the first half of its own S columns,
// so S_w(j+1) is issued after PV_w(j) (the tensor pipe runs one thread's MMAs in order, so it
// reads P before the next S lands there).  Issue order: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1).
// Either way the two warpgroups alternate: one computes exponentials while the tensor cores run the
// other's MMAs.  Heavy (late) tile pairs are scheduled first.  Every wait is bounded and unwinds on
// timeout.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pcb {
namespace fa {

constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kThreads = 384;  // warpgroups 0, 1: softmax; warpgroup 2: TMA warp, MMA warp, two idle warps
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512); warpgroup 2 drops to
// 96 (frees 4 x 32 x 72 = 9216), the softmax warpgroups rise to 200 (take 2 x 4 x 32 x 32 = 8192).
constexpr int kRegsCtl = 96;
constexpr int kRegsSoftmax = 200;
static_assert(4 * 32 * (2 * kRegsSoftmax + kRegsCtl) <= kThreads * 168, "register split exceeds the launch");
constexpr int kAtom = 128 * 128;  // bytes of one [128 rows x 64 bf16] swizzled atom
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // move the running max only when it grows by more than 2^8

// Optional cycle counters (build with -DPCB_ATTN_STATS), read with pcb_attn_fwd_stats():
//   0 softmax warp 0 loop   1 waits S   2 TMEM load of S   3 max / exp / pack   4 waits PV (P buffer free)
//   5 P store + arrive   6 O rescale   7 tiles   8 epilogue   9 MMA loop   10 MMA waits K/V   11 MMA waits
//   S read   12 MMA waits P   13 producer waits free stage
#ifdef PCB_ATTN_STATS
__device__ unsigned long long g_fwd_stats[16];
#define FST_T0(t) long long t = clock64()
#define FST_ADD(v, t) v += clock64() - t
#define FST_FLUSH(i, v) atomicAdd(&g_fwd_stats[i], (unsigned long long)(v))
#else
#define FST_T0(t)
#define FST_ADD(v, t)
#define FST_FLUSH(i, v)
#endif

template <int HD>
struct Cfg {
  static constexpr int ATOMS = HD / 64;
  static constexpr bool EARLY_S = HD == 64;                         // S released before P is written
  static constexpr int QBUF = HD == 64 ? 2 : 1;                     // Q buffers (tiles A, B each)
  static constexpr int STAGES = HD == 64 ? 3 : 2;                   // K/V ring depth
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QBUF * 2 * ATOMS * kAtom;
  static constexpr int V_OFF = K_OFF + STAGES * ATOMS * kAtom;
  static constexpr int BAR_OFF = V_OFF + STAGES * ATOMS * kAtom;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
  static constexpr int TM_S = 0;                                    // + w * 128
  static constexpr int TM_O = 2 * kBKV;                             // + w * HD
  static constexpr int TM_P = EARLY_S ? TM_O + 2 * HD : TM_S;       // + w * (EARLY_S ? 64 : 128)
  static constexpr int P_STRIDE = EARLY_S ? 64 : kBKV;
  static_assert(TM_O + 2 * HD <= 512 && (!EARLY_S || TM_P + 2 * 64 <= 512), "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

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

// Elementwise helpers of the softmax loop.  Exponentials and float->bf16 conversions share the SFU
// pipe (16 lanes per SM per clock), the busiest unit of the loop, so the conversions move to the ALU
// and the scale / row-sum arithmetic to paired fp32 instructions:
//  * pack_pos: two non-negative floats to a bf16 pair by adding half a bf16 ulp to the bit pattern and
//    keeping the high halves (round half up, which differs from round-to-nearest-even only on exact ties);
//  * ffma2 / fadd2: two fp32 lanes per instruction (fma.rn.f32x2 / add.rn.f32x2).
PCB_DEVICE uint32_t pack_pos(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}
PCB_DEVICE void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\t"
      "mov.b64 rc, {%5, %5};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
PCB_DEVICE void fadd2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, __nv_bfloat16* __restrict__ out, long long ld_o,
                       float* __restrict__ lse, int S, int H, int BH, float scale, int* err) {
  using C = Cfg<HD>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;                 // [2]
  uint64_t* q_empty = bars + 2;                // [2]
  uint64_t* kv_full = bars + 4;                // [ST]
  uint64_t* kv_empty = kv_full + ST;           // [ST]
  uint64_t* s_full = kv_empty + ST;            // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* o_final = p_full + 2;              // [2]
  uint64_t* s_free = o_final + 2;              // [2] (EARLY_S) softmax warpgroup w has S_w in registers
  uint64_t* pv_done = s_free + 2;              // [2] (EARLY_S) the PV MMA of warpgroup w has read P_w
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);
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
      mbar_init(&s_free[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < ST; ++i) {
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
  // programmatic dependent launch: barrier set-up and the TMEM allocation above overlap the previous
  // kernel's tail; no global memory is touched before it has completed
  pdl_wait();
  if (warp >= 8) {
    // control warpgroup: registers down, then the TMA warp and the MMA warp
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
    if (warp == 8 && lane == 0) {
      // ---------------- TMA producer: runs ahead into the next item ----------------
      int qc = 0, kc = 0;
      bool ok = true;
      long long st_pw = 0;
      (void)st_pw;
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++qc)) {
        const Item it = item_of(i, BH, T, H);
        const int qb = C::QBUF == 2 ? (qc & 1) : 0;
        const uint32_t qpar = C::QBUF == 2 ? (((qc >> 1) & 1) ^ 1u) : ((qc & 1) ^ 1u);
        if (!(ok = mbar_wait(&q_empty[qb], qpar, err, kErrTimeoutEmpty, abort_flag))) break;
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
          const int st = kc % ST;
          FST_T0(t0);
          if (!(ok = mbar_wait(&kv_empty[st], ((kc / ST) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
          FST_ADD(st_pw, t0);
          mbar_arrive_expect_tx(&kv_full[st], 2 * C::ATOMS * kAtom);
          const int krow = it.b * S + j * kBKV;
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a) {
            tma_load_2d(sK + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (H + it.h) * HD + a * 64, krow);
            tma_load_2d(sV + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (2 * H + it.h) * HD + a * 64, krow);
          }
        }
      }
      FST_FLUSH(13, st_pw);
    } else if (warp == 9 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16(kBQ, kBKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBQ, HD, 0, 1);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      long long st_kv = 0, st_sf = 0, st_pf = 0;
      (void)st_kv; (void)st_sf; (void)st_pf;
      FST_T0(st_loop);
      auto kv_ready = [&](int n) -> bool {
        FST_T0(t0);
        const bool r = mbar_wait(&kv_full[n % ST], (n / ST) & 1, err, kErrTimeoutFull, abort_flag);
        FST_ADD(st_kv, t0);
        return r;
      };
      int n_s[2] = {0, 0}, n_pv[2] = {0, 0};     // S / PV MMAs issued per warpgroup (phase counters)
      auto issue_s = [&](int w, int qb, int n) -> bool {
        FST_T0(t0);
        if (C::EARLY_S && n_s[w] > 0 &&
            !mbar_wait(&s_free[w], (n_s[w] - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag))
          return false;
        FST_ADD(st_sf, t0);
        ++n_s[w];
        const uint32_t kb = k_addr + (n % ST) * C::ATOMS * kAtom;
        const uint32_t qa = q_addr + (qb * 2 + w) * C::ATOMS * kAtom;
        const uint64_t ad = make_smem_desc(qa, 16, 1024, 2), bd = make_smem_desc(kb, 16, 1024, 2);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {  // advancing the start address = adding (bytes >> 4) to the descriptor
          const uint64_t off = ((k >> 2) * kAtom + (k & 3) * 32) >> 4;
          umma_bf16(tmem + C::TM_S + w * kBKV, ad + off, bd + off, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
        return true;
      };
      auto issue_pv = [&](int w, int n, bool first) -> bool {  // A = P from TMEM (16 keys = 8 columns per step)
        FST_T0(t0);
        if (!mbar_wait(&p_full[w], n_pv[w] & 1, err, kErrTimeoutTmemEmpty, abort_flag)) return false;
        FST_ADD(st_pf, t0);
        ++n_pv[w];
        const uint32_t vb = v_addr + (n % ST) * C::ATOMS * kAtom;
        const uint64_t bd = make_smem_desc(vb, kAtom, 1024, 2);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBKV / 16; ++k)
          umma_bf16_ts(tmem + C::TM_O + w * HD, tmem + C::TM_P + w * C::P_STRIDE + k * 8, bd + (k * 2048 >> 4),
                       idesc_o, (!first || k > 0) ? 1u : 0u);
        if (C::EARLY_S) umma_commit(&pv_done[w]);
        return true;
      };
      int qc = 0, kc = 0;
      bool ok = true;
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++qc)) {
        const Item it = item_of(i, BH, T, H);
        const int qb = C::QBUF == 2 ? (qc & 1) : 0;
        const uint32_t qpar = C::QBUF == 2 ? ((qc >> 1) & 1) : (qc & 1);
        const int last_a = 2 * it.t, n_kv = 2 * it.t + 2;
        // S_w(0) may overwrite S_w: (EARLY_S) the s_free wait inside issue_s; (otherwise) the previous
        // item's last p_full_w, waited below, proved the softmax had read it
        if (!(ok = mbar_wait(&q_full[qb], qpar, err, kErrTimeoutFull, abort_flag) && kv_ready(kc))) break;
        if (!(ok = issue_s(0, qb, kc) && issue_s(1, qb, kc))) break;
        for (int j = 0; j < n_kv && ok; ++j) {
          const int n = kc + j;
          if (C::EARLY_S) {
            if (j + 1 < n_kv) {
              if (!(ok = kv_ready(n + 1))) break;
              if (j + 1 <= last_a && !(ok = issue_s(0, qb, n + 1))) break;
              if (!(ok = issue_s(1, qb, n + 1))) break;
            }
            if (j <= last_a) {
              if (!(ok = issue_pv(0, n, j == 0))) break;
              if (j == last_a) umma_commit(&o_final[0]);
            }
            if (!(ok = issue_pv(1, n, j == 0))) break;
            umma_commit(&kv_empty[n % ST]);
            if (j + 1 == n_kv) {
              umma_commit(&q_empty[qb]);
              umma_commit(&o_final[1]);
            }
          } else {
            if (j <= last_a) {
              if (!(ok = issue_pv(0, n, j == 0))) break;
              if (j + 1 <= last_a) {
                if (!(ok = kv_ready(n + 1) && issue_s(0, qb, n + 1))) break;
              } else {
                umma_commit(&o_final[0]);
              }
            }
            if (!(ok = issue_pv(1, n, j == 0))) break;
            umma_commit(&kv_empty[n % ST]);
            if (j + 1 < n_kv) {
              if (!(ok = kv_ready(n + 1) && issue_s(1, qb, n + 1))) break;
            } else {
              umma_commit(&q_empty[qb]);
              umma_commit(&o_final[1]);
            }
          }
        }
        kc += n_kv;
      }
      FST_FLUSH(9, clock64() - st_loop);
      FST_FLUSH(10, st_kv);
      FST_FLUSH(11, st_sf);
      FST_FLUSH(12, st_pf);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ---------------- softmax warpgroups: one query row per thread ----------------
    const int w = warp >> 2;                    // 0 = tile A, 1 = tile B
    const int r = threadIdx.x & 127;            // row within the tile == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = lane_base + C::TM_S + w * kBKV;
    const uint32_t o_col = lane_base + C::TM_O + w * HD;
    const uint32_t p_col = lane_base + C::TM_P + w * C::P_STRIDE;
    const float c = scale * kLog2e;
    int tc = 0, ic = 0;
    bool ok = true;
    long long sx[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    (void)sx;
    FST_T0(sx_loop);
    for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
      const Item it = item_of(i, BH, T, H);
      const int last = 2 * it.t + w;           // tile A: key tiles 0..2t, tile B: 0..2t+1
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j <= last; ++j, ++tc) {
        FST_T0(t1);
        ok = mbar_wait(&s_full[w], tc & 1, err, kErrTimeoutTmemFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        FST_ADD(sx[1], t1);
        tc_fence_after();
        FST_T0(t2);
        uint32_t sv_u[128];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          tmem_ld_32x32b_x32(s_col + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(sv_u + cc * 32));
        tmem_ld_wait();
        FST_ADD(sx[2], t2);
        FST_T0(t3);
        if (C::EARLY_S) {  // S_w is in registers: the next S_w MMA may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[w]);
        }
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
        if constexpr (C::EARLY_S) {
          // all of P in registers first; it may be stored only after PV_w of the previous tile read P_w
          uint32_t pk[64];
#pragma unroll
          for (int e = 0; e < 128; e += 2) {
            float x0, x1;
            ffma2(x0, x1, SV(e), SV(e + 1), c, -msc);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            fadd2(rsv[(e >> 1) & 1], rsv[((e >> 1) & 1) + 2], p0, p1);
            pk[e >> 1] = pack_pos(p0, p1);
          }
          FST_ADD(sx[3], t3);
          FST_T0(t4);
          if (tc > 0) {
            ok = mbar_wait(&pv_done[w], (tc - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            tc_fence_after();
          }
          FST_ADD(sx[4], t4);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            tmem_st_32x32b_x16(p_col + q4 * 16, *reinterpret_cast<const uint32_t(*)[16]>(pk + q4 * 16));
        } else {
          // P over its own S columns, a quarter at a time (S is already in registers)
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float x0, x1;
              ffma2(x0, x1, SV(q4 * 32 + e), SV(q4 * 32 + e + 1), c, -msc);
              const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
              fadd2(rsv[(e >> 1) & 1], rsv[((e >> 1) & 1) + 2], p0, p1);
              pk[e >> 1] = pack_pos(p0, p1);
            }
            tmem_st_32x32b_x16(p_col + q4 * 16, pk);
          }
        }
#undef SV
        l += (rsv[0] + rsv[1]) + (rsv[2] + rsv[3]);
        FST_T0(t6);
        if (rescale && j > 0) {  // O holds PV(0..j-1): scale it in place (PV_w(j-1) is complete)
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
        FST_ADD(sx[6], t6);
        FST_T0(t5);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[w]);
        FST_ADD(sx[5], t5);
        ++sx[7];
      }
      if (!ok) break;
      FST_T0(t8);
      ok = mbar_wait(&o_final[w], ic & 1, err, kErrTimeoutTmemFull, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      // epilogue: the next item's PV_w(0) overwrites O_w only after this warpgroup's next p_full_w,
      // which it signals after these loads completed
      const int q = it.t * 2 * kBQ + w * kBQ + r;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (long long)(it.b * S + q) * ld_o + it.h * HD;
#pragma unroll 1
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
      FST_ADD(sx[8], t8);
    }
    if (threadIdx.x == 0) {
      FST_FLUSH(0, clock64() - sx_loop);
      for (int k = 1; k < 9; ++k) FST_FLUSH(k, sx[k]);
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
  step_launch(fa::attn_fwd_tc_kernel<HD>, dim3(grid), dim3(fa::kThreads), C::SMEM, s, tm,
             reinterpret_cast<__nv_bfloat16*>(out), ld_o, lse, S, H, B * H, scale, err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(1000 + static_cast<int>(e));
}

}  // namespace pcb

// Copies the forward's cycle counters into out[16] and clears them; -1 when built without them.
int pcb_attn_fwd_stats(unsigned long long* out) {
#ifdef PCB_ATTN_STATS
  if (cudaMemcpyFromSymbol(out, pcb::fa::g_fwd_stats, 16 * sizeof(unsigned long long)) != cudaSuccess) return -2;
  unsigned long long zero[16] = {};
  cudaMemcpyToSymbol(pcb::fa::g_fwd_stats, zero, sizeof(zero));
  return 0;
#else
  (void)out;
  return -1;
#endif
}

// Same contract as pcb_attn_fwd (qkv [B*S, 3*H*HD] bf16 with q|k|v column blocks, out [B*S, H*HD]
// bf16, lse [B*H, S] fp32), on tcgen05.  S % 256 == 0, HD 64 or 128, row strides % 8 == 0.
int pcb_attn_fwd_tc(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                    int HD, float scale, int* err, cudaStream_t s) {
  if (S % 256 != 0 || ld % 8 || ld_o % 8) return -1;
  if (reinterpret_cast<uintptr_t>(qkv) & 15) return -1;
  if (HD == 64) return pcb::fa_launch<64>(qkv, ld, out, ld_o, lse, B, S, H, scale, err, s);
  if (HD == 128) return pcb::fa_launch<128>(qkv, ld, out, ld_o, lse, B, S, H, scale, err, s);
  return -1;
}
