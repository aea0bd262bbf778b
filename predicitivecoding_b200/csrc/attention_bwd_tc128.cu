// Causal flash-attention backward on tcgen05 for head dim 128.
//
// Reference counterpart: PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs (attn_bwd_dq,
// attn_bwd_dkv: fp32 SIMT, P replayed from the logsumexp).  Same plan as the head-dim-64 kernel
// (persistent CTAs over 128-key tiles, keys on the TMEM lanes, P^T as the TMEM operand of dV, dS^T in
// shared memory serving two MMAs) with the tile shapes changed so that every accumulator fits the
// 512 TMEM columns at head dim 128:
//   query tiles of 64:   S^T  = K Q_i^T     M=128 keys, N=64 queries, K=128        -> TMEM S   (64 cols)
//                        dP^T = V dO_i^T    same                                     -> TMEM dP  (64 cols)
//   gradient warpgroups: P^T = 2^(S^T c - lse log2 e), causal mask, dS^T = P^T (dP^T - D); P^T to TMEM
//                        as bf16 (32 cols), dS^T to shared memory (one 128-row swizzled atom)
//                        dV  += P^T dO_i    M=128 keys, N=128 head dims, K=64        -> TMEM dV  (128)
//                        dK  += dS^T Q_i    same                                      -> TMEM dK  (128)
//   transposed dQ:       dQ_i^T = K^T dS^T  M=128 head dims, N=64 queries, K=128 keys -> TMEM dQT (64)
//   dQ warpgroup: thread = head dim; dQ^T * scale staged as four [64 x 32] fp32 boxes (a warp writes 32
//   consecutive floats of one query row: no bank conflicts) and added to the fp32 accumulator with
//   TMA reduce-add.
// TMEM: S 64 + dP 64 + P 32 + dV 128 + dK 128 + dQT 64 = 480 columns.  Every wait is bounded.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pcb {
namespace fab128 {

constexpr int kKT = 128;          // keys per item
constexpr int kQT = 64;           // queries per tile
constexpr int kHD = 128;
constexpr int kThreads = 512;     // WG0/WG1 gradient (queries 0-31 / 32-63), WG2 dQ, warp 12 TMA, warp 13 MMA
constexpr int kTmaWarp = 12, kMmaWarp = 13;
constexpr int kRegsCtl = 80, kRegsDq = 96, kRegsGrad = 168;
static_assert(4 * 32 * (2 * kRegsGrad + kRegsDq + kRegsCtl) <= kThreads * 128, "register split exceeds the launch");
constexpr int kAtom = 128 * 128;  // [128 rows x 64 bf16], 128-byte swizzle
constexpr int kHalf = 64 * 128;   // [64 rows x 64 bf16]
constexpr float kLog2e = 1.4426950408889634f;

constexpr int kQStages = 3;
constexpr int K_OFF = 0;                              // 2 atoms (head dims 0-63, 64-127)
constexpr int V_OFF = K_OFF + 2 * kAtom;              // 2 atoms
constexpr int Q_OFF = V_OFF + 2 * kAtom;              // kQStages x 2 half atoms
constexpr int DO_OFF = Q_OFF + kQStages * 2 * kHalf;  // kQStages x 2 half atoms
constexpr int DS_OFF = DO_OFF + kQStages * 2 * kHalf; // 2 buffers x 1 atom
constexpr int DQ_OFF = DS_OFF + 2 * kAtom;            // 4 boxes of [64 rows x 32 fp32] (8 KB each)
constexpr int BAR_OFF = DQ_OFF + 4 * 8192;
constexpr int SMEM = BAR_OFF + 256 + 1024;
static_assert(SMEM <= 232448, "shared memory budget");

constexpr int TM_S = 0, TM_DP = 64, TM_P = 128, TM_DV = 160, TM_DK = 288, TM_DQ = 416;
static_assert(TM_DQ + kQT <= 512, "TMEM budget");

struct Item {
  int kb, b, h, bh;
};
PCB_DEVICE Item item_of(int i, int BH, int H) {
  Item it;
  it.kb = i / BH;
  it.bh = i % BH;
  it.b = it.bh / H;
  it.h = it.bh % H;
  return it;
}

PCB_DEVICE void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
PCB_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
PCB_DEVICE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
PCB_DEVICE void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
PCB_DEVICE void dq_wg_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
PCB_DEVICE bool dq_wg_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_tc128_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_dq,
                          const float* __restrict__ lse, const float* __restrict__ dvec,
                          __nv_bfloat16* __restrict__ dqkv, long long ld_d, int S, int H, float scale,
                          const float2* __restrict__ rope_cs, int BH, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + K_OFF;
  uint8_t* sV = smem + V_OFF;
  uint8_t* sQ = smem + Q_OFF;
  uint8_t* sDO = smem + DO_OFF;
  uint8_t* sDS = smem + DS_OFF;
  uint8_t* sDQ = smem + DQ_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_empty = bars + 1;
  uint64_t* ld_full = bars + 2;    // [kQStages]
  uint64_t* ld_empty = bars + 5;   // [kQStages]
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 9;
  uint64_t* ds_full = bars + 10;
  uint64_t* p_done = bars + 11;
  uint64_t* dq_full = bars + 12;
  uint64_t* dq_empty = bars + 13;
  uint64_t* acc_full = bars + 14;
  uint64_t* grad_done = bars + 15;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TK = S / kKT;      // key tiles
  const int TQ = S / kQT;      // query tiles
  const int n_items = TK * BH;
  const int D = H * kHD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(&ld_full[i], 1);
      mbar_init(&ld_empty[i], 1 + 8);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&grad_done[i], 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(ds_full, 8);
    mbar_init(p_done, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&tm_kv);
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_do);
  }
  if (warp == kMmaWarp) {
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

  if (warp >= 12) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
    if (warp == kTmaWarp && lane == 0) {
      // ---------------- TMA producer ----------------
      int ic = 0, lc = 0;
      bool ok = true;
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
        const Item it = item_of(i, BH, H);
        if (!(ok = mbar_wait(kv_empty, (ic & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
        mbar_arrive_expect_tx(kv_full, 4 * kAtom);
        const int krow = it.b * S + it.kb * kKT;
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          tma_load_2d(sK + a * kAtom, &tm_kv, kv_full, (H + it.h) * kHD + a * 64, krow);
          tma_load_2d(sV + a * kAtom, &tm_kv, kv_full, (2 * H + it.h) * kHD + a * 64, krow);
        }
        for (int qi = 2 * it.kb; qi < TQ; ++qi, ++lc) {
          const int st = lc % kQStages;
          if (!(ok = mbar_wait(&ld_empty[st], ((lc / kQStages) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
          mbar_arrive_expect_tx(&ld_full[st], 4 * kHalf);
          const int qrow = it.b * S + qi * kQT;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            tma_load_2d(sQ + (st * 2 + a) * kHalf, &tm_q, &ld_full[st], it.h * kHD + a * 64, qrow);
            tma_load_2d(sDO + (st * 2 + a) * kHalf, &tm_do, &ld_full[st], it.h * kHD + a * 64, qrow);
          }
        }
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16(128, kQT, 0, 0);   // S^T, dP^T: K-major operands
      constexpr uint32_t idesc_v = make_idesc_bf16(128, kHD, 0, 1);   // dV: A TMEM, B MN-major
      constexpr uint32_t idesc_k = make_idesc_bf16(128, kHD, 0, 1);   // dK: A K-major, B MN-major
      constexpr uint32_t idesc_q = make_idesc_bf16(128, kQT, 1, 1);   // dQ^T: A M-major, B MN-major
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ), do_addr = smem_u32(sDO),
                     ds_addr = smem_u32(sDS);
      int ic = 0, lc = 0, tcount = 0;
      bool ok = true;
      auto grad = [&](int v, int st, bool first) -> bool {  // dV, dK, dQ^T of the tile with counter v
        if (!mbar_wait(ds_full, v & 1, err, kErrTimeoutTmemEmpty, abort_flag)) return false;
        tc_fence_after();
        const uint64_t bdo = make_smem_desc(do_addr + st * 2 * kHalf, kHalf, 1024, 2);
        const uint64_t bq = make_smem_desc(q_addr + st * 2 * kHalf, kHalf, 1024, 2);
        const uint32_t dsb = ds_addr + (v & 1) * kAtom;
#pragma unroll
        for (int k = 0; k < kQT / 16; ++k)  // dV += P^T dO_i (16 queries = 8 TMEM columns per step)
          umma_bf16_ts(tmem + TM_DV, tmem + TM_P + k * 8, bdo + (k * 2048 >> 4), idesc_v, (!first || k > 0) ? 1u : 0u);
        umma_commit(p_done);
        const uint64_t ads = make_smem_desc(dsb, 16, 1024, 2);
#pragma unroll
        for (int k = 0; k < kQT / 16; ++k)  // dK += dS^T Q_i
          umma_bf16(tmem + TM_DK, ads + ((k * 32) >> 4), bq + (k * 2048 >> 4), idesc_k, (!first || k > 0) ? 1u : 0u);
        if (v > 0 && !mbar_wait(dq_empty, (v - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag)) return false;
        tc_fence_after();
        const uint64_t ak = make_smem_desc(k_addr, kAtom, 1024, 2);     // K read head-dim-major
        const uint64_t bds = make_smem_desc(dsb, kAtom, 1024, 2);        // dS^T read query-major
#pragma unroll
        for (int k = 0; k < kKT / 16; ++k)  // dQ^T = K^T dS^T over the 128 keys
          umma_bf16(tmem + TM_DQ, ak + (k * 2048 >> 4), bds + (k * 2048 >> 4), idesc_q, k > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&grad_done[v & 1]);
        umma_commit(&ld_empty[st]);
        return true;
      };
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
        const Item it = item_of(i, BH, H);
        if (!(ok = mbar_wait(kv_full, ic & 1, err, kErrTimeoutFull, abort_flag))) break;
        const uint64_t ak = make_smem_desc(k_addr, 16, 1024, 2), av = make_smem_desc(v_addr, 16, 1024, 2);
        int prev_st = 0;
        for (int qi = 2 * it.kb; qi < TQ && ok; ++qi, ++lc, ++tcount) {
          const int st = lc % kQStages;
          if (!(ok = mbar_wait(&ld_full[st], (lc / kQStages) & 1, err, kErrTimeoutFull, abort_flag))) break;
          if (tcount > 0 && !(ok = mbar_wait(s_free, (tcount - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag))) break;
          tc_fence_after();
          const uint64_t bq = make_smem_desc(q_addr + st * 2 * kHalf, 16, 1024, 2);
          const uint64_t bdo = make_smem_desc(do_addr + st * 2 * kHalf, 16, 1024, 2);
#pragma unroll
          for (int k = 0; k < kHD / 16; ++k) {  // S^T = K Q_i^T, dP^T = V dO_i^T over the 128 head dims
            const uint64_t oa = ((k >> 2) * kAtom + (k & 3) * 32) >> 4;
            const uint64_t ob = ((k >> 2) * kHalf + (k & 3) * 32) >> 4;
            umma_bf16(tmem + TM_S, ak + oa, bq + ob, idesc_s, k > 0 ? 1u : 0u);
            umma_bf16(tmem + TM_DP, av + oa, bdo + ob, idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(s_full);
          if (qi > 2 * it.kb && !(ok = grad(tcount - 1, prev_st, qi - 1 == 2 * it.kb))) break;
          prev_st = st;
        }
        if (!ok) break;
        if (!(ok = grad(tcount - 1, prev_st, TQ - 1 == 2 * it.kb))) break;
        umma_commit(acc_full);
        umma_commit(kv_empty);
      }
    }
  } else if (warp < 8) {
    // ---------------- gradient warpgroups: thread = key row = TMEM lane; gw owns queries 32gw.. ----------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsGrad));
    const int gw = warp >> 2;
    const int r = threadIdx.x & 127;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float cl = scale * kLog2e;
    int lc = 0, tcount = 0, ic = 0;
    bool ok = true;
    for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
      const Item it = item_of(i, BH, H);
      for (int qi = 2 * it.kb; qi < TQ; ++qi, ++lc, ++tcount) {
        const int st = lc % kQStages;
        ok = mbar_wait(&ld_full[st], (lc / kQStages) & 1, err, kErrTimeoutFull, abort_flag) &&
             mbar_wait(s_full, tcount & 1, err, kErrTimeoutTmemFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const float* sl = lse + (long long)it.bh * S + qi * kQT + 32 * gw;
        const float* sd = dvec + (long long)it.bh * S + qi * kQT + 32 * gw;
        // key r is visible to query column q of this tile iff r <= q + 64 * (qi - 2 kb)
        const int lim = r - 64 * (qi - 2 * it.kb);
        {   // pull the next tile's lse / delta line (this warpgroup's 32 queries) into L1 meanwhile
          int nbh = it.bh, nq = qi + 1;
          if (nq >= TQ) {
            const int ni = snake_item(ic + 1);
            nbh = ni < n_items ? ni % BH : -1;
            nq = ni < n_items ? 2 * (ni / BH) : 0;
          }
          if (nbh >= 0 && lane < 2)
            prefetch_l1((lane == 0 ? lse : dvec) + (long long)nbh * S + nq * kQT + 32 * gw);
        }
        // this warpgroup's 32 query columns in two chunks of 16: chunk 1's TMEM and L1 loads are in flight
        // while chunk 0 is finished
        uint32_t su[2][16], du[2][16];
        float lv[2][16], dv[2][16];
        auto fetch = [&](int c, int b) {
          tmem_ld_32x32b_x16(lane_base + TM_S + 32 * gw + 16 * c, su[b]);
          tmem_ld_32x32b_x16(lane_base + TM_DP + 32 * gw + 16 * c, du[b]);
#pragma unroll
          for (int e = 0; e < 16; e += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(sl + 16 * c + e);
            const float4 d4 = *reinterpret_cast<const float4*>(sd + 16 * c + e);
            lv[b][e] = -l4.x * kLog2e;
            lv[b][e + 1] = -l4.y * kLog2e;
            lv[b][e + 2] = -l4.z * kLog2e;
            lv[b][e + 3] = -l4.w * kLog2e;
            dv[b][e] = -d4.x;
            dv[b][e + 1] = -d4.y;
            dv[b][e + 2] = -d4.z;
            dv[b][e + 3] = -d4.w;
          }
        };
        fetch(0, 0);
        fetch(1, 1);
        tmem_ld_wait_regs(su[0], du[0]);
        tmem_ld_wait_regs(su[1], du[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);   // S/dP of this warp are in registers: the next tile's MMAs may start
        // P of the previous tile must have been read by its dV MMA; this dS buffer by the MMAs two tiles back
        if (tcount > 0) ok = mbar_wait(p_done, (tcount - 1) & 1, err, kErrTimeoutTmemFull, abort_flag);
        if (ok && tcount > 1)
          ok = mbar_wait(&grad_done[tcount & 1], ((tcount - 2) >> 1) & 1, err, kErrTimeoutTmemFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        // dS^T row r: 16-byte chunk j (8 queries) at ((j ^ (r & 7)) << 4); this warpgroup owns chunks 4gw..4gw+3
        uint8_t* drow = sDS + (tcount & 1) * kAtom + r * 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[8], dk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const int q = 32 * gw + 16 * c + e;
            float x0, x1, p0, p1, g0, g1;
            ffma2v(x0, x1, __uint_as_float(su[c][e]), __uint_as_float(su[c][e + 1]), cl, lv[c][e], lv[c][e + 1]);
            p0 = q >= lim ? ex2_approx(x0) : 0.f;
            p1 = q + 1 >= lim ? ex2_approx(x1) : 0.f;
            fmul_add2(g0, g1, p0, p1, __uint_as_float(du[c][e]), __uint_as_float(du[c][e + 1]), dv[c][e],
                      dv[c][e + 1]);
            pk[e >> 1] = pack_bf16_alu(p0, p1);
            dk[e >> 1] = pack_bf16_alu(g0, g1);
          }
          tmem_st_32x32b_x8(lane_base + TM_P + 16 * gw + 8 * c, pk);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int chunk = 4 * gw + 2 * c + h;
            *reinterpret_cast<uint4*>(drow + ((chunk ^ (r & 7)) << 4)) =
                make_uint4(dk[4 * h], dk[4 * h + 1], dk[4 * h + 2], dk[4 * h + 3]);
          }
        }
        tmem_st_wait();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(ds_full);
          mbar_arrive(&ld_empty[st]);
        }
      }
      if (!ok) break;
      // ---- dK, dV of this key tile: warpgroup 0 writes dK * scale (rotated back by -theta with a RoPE
      // table), warpgroup 1 writes dV ----
      ok = mbar_wait(acc_full, ic & 1, err, kErrTimeoutTmemFull, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const long long row = (long long)it.b * S + it.kb * kKT + r;
      __nv_bfloat16* dst = dqkv + row * ld_d + (gw == 0 ? D : 2 * D) + it.h * kHD;
      const float mul = gw == 0 ? scale : 1.f;
      const bool rot = gw == 0 && rope_cs != nullptr;
      const int pos = it.kb * kKT + r;
#pragma unroll 1
      for (int cc = 0; cc < kHD / 32; ++cc) {
        uint32_t u32[32];
        tmem_ld_32x32b_x32(lane_base + (gw == 0 ? TM_DK : TM_DV) + cc * 32, u32);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          float kv[8];
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            float a0 = __uint_as_float(u32[e + u]) * mul, a1 = __uint_as_float(u32[e + u + 1]) * mul;
            if (rot) {
              const float2 cs = rope_cs[pos * (kHD / 2) + ((cc * 32 + e + u) >> 1)];
              const float b0 = a0 * cs.x + a1 * cs.y, b1 = -a0 * cs.y + a1 * cs.x;
              a0 = b0;
              a1 = b1;
            }
            kv[u] = a0;
            kv[u + 1] = a1;
          }
          *reinterpret_cast<uint4*>(dst + cc * 32 + e) =
              make_uint4(pack_bf16x2(kv[0], kv[1]), pack_bf16x2(kv[2], kv[3]), pack_bf16x2(kv[4], kv[5]),
                         pack_bf16x2(kv[6], kv[7]));
        }
      }
      tc_fence_before();
    }
  } else {
    // ---------------- dQ warpgroup: thread = head dim = TMEM lane ----------------
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsDq));
    const int d = threadIdx.x - 256;               // head dim 0..127
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    int tcount = 0;
    bool ok = true;
    for (int ic = 0, i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
      const Item it = item_of(i, BH, H);
      for (int qi = 2 * it.kb; qi < TQ; ++qi, ++tcount) {
        ok = dq_wg_all(mbar_wait(dq_full, tcount & 1, err, kErrTimeoutTmemFull, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (d == 0) bulk_wait_read0();   // the previous tile's reductions have read the staging boxes
        dq_wg_sync();
        // box (d / 32): [64 query rows x 32 dims], 128-byte rows; 16-byte chunk j of row q at ((j ^ (q & 7)) << 4)
        uint8_t* box = sDQ + (d >> 5) * 8192;
        const int col = d & 31;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t qu[32];
          tmem_ld_32x32b_x32(lane_base + TM_DQ + 32 * half, qu);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int q = 32 * half + j;
            *reinterpret_cast<float*>(box + q * 128 + (((col >> 2) ^ (q & 7)) << 4) + (col & 3) * 4) =
                __uint_as_float(qu[j]) * scale;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        dq_wg_sync();
        if (d == 0) {
          const int y = it.b * S + qi * kQT;
#pragma unroll
          for (int bx = 0; bx < 4; ++bx) tma_reduce_add_2d(&tm_dq, sDQ + bx * 8192, it.h * kHD + 32 * bx, y);
          bulk_commit();
        }
      }
    }
    if (d == 0) bulk_wait0();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

// delta[b*H + h][i] = sum_d dO[row, h, d] * O[row, h, d]: 16 lanes per (row, head), 16-byte loads;
// and zeroes the fp32 dQ accumulator (n4 float4s) in the same pass, which the backward kernel adds into
__global__ void bwd_delta128_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                    long long ld_o, float* __restrict__ dvec, long long rows_h, int S, int H,
                                    float4* __restrict__ dq_zero, long long n4) {
  pdl_wait();
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
    dq_zero[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < rows_h * 16; t += stride) {
    const long long hr = t >> 4;
    const int part = (int)(t & 15);
    const long long row = hr / H;
    const int h = (int)(hr % H);
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * ld_o + h * kHD + part * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + row * ld_o + h * kHD + part * 8);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc += bf16_lo(av[k]) * bf16_lo(gv[k]) + bf16_hi(av[k]) * bf16_hi(gv[k]);
#pragma unroll
    for (int o2 = 1; o2 < 16; o2 <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
    if (part == 0) dvec[((row / S) * H + h) * S + row % S] = acc;
  }
}

// dqkv[:, 0:D] = bf16(dq_acc) (rotated by -theta with a RoPE table): 8 values per thread
__global__ void bwd_dq_convert128_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv,
                                         long long ld_d, long long rows, int D, int S,
                                         const float2* __restrict__ rope_cs) {
  pdl_wait();
  const long long per_row = D / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < rows * per_row; t += stride) {
    const long long r = t / per_row;
    const int c = (int)(t % per_row) * 8;
    const float4 x0 = *reinterpret_cast<const float4*>(dq_acc + r * D + c);
    const float4 x1 = *reinterpret_cast<const float4*>(dq_acc + r * D + c + 4);
    float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    if (rope_cs != nullptr) {
      const float2* cs = rope_cs + (r % S) * (kHD / 2) + ((c % kHD) >> 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 q = cs[k];
        const float a = v[2 * k], b = v[2 * k + 1];
        v[2 * k] = a * q.x + b * q.y;
        v[2 * k + 1] = -a * q.y + b * q.x;
      }
    }
    *reinterpret_cast<uint4*>(dqkv + r * ld_d + c) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                                pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

}  // namespace fab128

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_fab128() {
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

static bool encode_map(PFN_cuTensorMapEncodeTiled_v12000 fn, CUtensorMap* tm, const void* base,
                       CUtensorMapDataType dt, int elt, long long cols, long long rows, long long ld, uint32_t bx,
                       uint32_t by) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * elt};
  cuuint32_t box[2] = {bx, by};
  cuuint32_t es[2] = {1, 1};
  return fn(tm, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace pcb

// Same contract as pcb_attn_bwd_rope, on tcgen05 for head dim 128: S % 128 == 0, row strides % 8 == 0,
// 16-byte aligned operands.  Returns 0, -1 (unsupported), -5 (tensor-map encode) or -(1000 + cudaError).
int pcb_attn_bwd_tc128(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                       const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                       float scale, const float* rope_cs, int* err, cudaStream_t s) {
  using namespace pcb;
  constexpr int HD = fab128::kHD;
  if (S % 128 != 0 || ld % 8 || ld_o % 8 || ld_d % 8) return -1;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(lse) | reinterpret_cast<uintptr_t>(dvec) | reinterpret_cast<uintptr_t>(dq_acc) |
       reinterpret_cast<uintptr_t>(dqkv)) & 15)
    return -1;
  auto fn = encode_fn_fab128();
  if (!fn) return -5;
  CUtensorMap tkv, tq, tdo, tdq;
  const long long rows = (long long)B * S;
  if (!encode_map(fn, &tkv, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3LL * H * HD, rows, ld, 64, 128) ||
      !encode_map(fn, &tq, qkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3LL * H * HD, rows, ld, 64, 64) ||
      !encode_map(fn, &tdo, dout, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (long long)H * HD, rows, ld_o, 64, 64) ||
      !encode_map(fn, &tdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (long long)H * HD, rows, (long long)H * HD, 32,
                  64))
    return -5;
  step_launch(fab128::bwd_delta128_kernel, dim3(148 * 8), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(out),
             reinterpret_cast<const __nv_bfloat16*>(dout), ld_o, dvec, rows * H, S, H,
             reinterpret_cast<float4*>(dq_acc), rows * H * HD / 4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fab128::attn_bwd_tc128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fab128::SMEM);
    attr = true;
  }
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_sms <= 0) num_sms = 148;
  }
  const int n_items = B * H * (S / fab128::kKT);
  const int grid = n_items < num_sms ? n_items : num_sms;
  step_launch(fab128::attn_bwd_tc128_kernel, dim3(grid), dim3(fab128::kThreads), fab128::SMEM, s, tkv, tq, tdo, tdq,
             lse, dvec, reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d, S, H, scale,
             reinterpret_cast<const float2*>(rope_cs), B * H, err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return -(1000 + static_cast<int>(e));
  step_launch(fab128::bwd_dq_convert128_kernel, dim3(148 * 8), dim3(256), 0, s, dq_acc,
             reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d, rows, H * HD, S, reinterpret_cast<const float2*>(rope_cs));
  const cudaError_t e2 = cudaGetLastError();
  return e2 == cudaSuccess ? 0 : -(1000 + static_cast<int>(e2));
}
