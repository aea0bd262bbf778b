// Causal flash-attention backward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference counterpart: PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs (attn_bwd_dq,
// attn_bwd_dkv: one block per query / per key, fp32 SIMT, P replayed from the logsumexp).
//
// Work item = one 128-key tile (kb) of one (batch, head); persistent CTAs walk the items heaviest
// first (kb = 0 sees every query tile).  For each query tile i >= kb the CTA computes, with the
// keys on the TMEM lanes:
//   (1) S^T  = K Q_i^T          M=128 keys, N=128 queries, K=hd     -> TMEM S
//   (2) dP^T = V dO_i^T         M=128 keys, N=128 queries, K=hd     -> TMEM dP
//   gradient warpgroup: P^T = 2^(S^T c - lse_i log2 e) (c = scale log2 e), causal mask on the
//       diagonal tile, dS^T = P^T (dP^T - D_i); P^T goes back to TMEM as bf16 (the A operand of
//       (3)), dS^T to shared memory in the 128B-swizzled layout that is K-major for (4) and
//       M-major for (5)
//   (3) dV  += P^T dO_i         A = P^T from TMEM, B = dO_i (MN-major)
//   (4) dK  += dS^T Q_i         A = dS^T (K-major), B = Q_i (MN-major)
//   (5) dQ_i = dS K             A = dS^T read M-major, B = K (MN-major) -> TMEM dQ
//   dQ warpgroup: dQ_i * scale is added to the fp32 accumulator with vector reductions.
// Two gradient warpgroups share the elementwise work (query columns 0-63 and 64-127).  After the
// last query tile they write dK * scale (rotated back by -theta when a RoPE table is given) and dV
// in bf16.  dS^T is double-buffered in shared memory, so a tile's gradient math waits only for the
// previous tile's dV MMA (which read P) before storing.  TMEM: S 128 + dP 128 + P 64 + dV 64 + dK 64 + dQ 64 = 512
// columns, no aliasing.  The MMA thread issues S/dP of tile i+1 as soon as the gradient warpgroup
// has read S/dP of tile i, so those MMAs overlap the elementwise work; every other hazard is
// covered by a commit that follows the MMAs it protects.  Every wait is bounded.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pcb {
namespace fab {

// Optional cycle counters (build with -DPCB_ATTN_STATS), read with pcb_attn_bwd_stats():
//   0 MMA issuer loop   1 MMA waits Q/dO stage   2 MMA waits S/dP read (s_free)   3 MMA waits dS (ds_full)
//   4 MMA waits dQ drained   5 gradient warp 0: waits stage + S/dP   6 gradient warp 0: waits P read / dS buffer
//   7 gradient warp 0 loop   8 dQ warp: waits dQ   9 dQ warp: waits staging reads   10 dQ warp loop
//   11 producer waits free stage   12 gradient warp 0 waits dK/dV   13 tiles issued by the MMA warps
#ifdef PCB_ATTN_STATS
__device__ unsigned long long g_attn_stats[16];
#define AST_DECL(v) long long v = 0
#define AST_T0(t) const long long t = clock64()
#define AST_ADD(v, t) v += clock64() - t
#define AST_FLUSH(i, v) atomicAdd(&g_attn_stats[i], (unsigned long long)(v))
#else
#define AST_DECL(v)
#define AST_T0(t)
#define AST_ADD(v, t)
#define AST_FLUSH(i, v)
#endif

constexpr int kT = 128;            // keys per item, queries per tile
constexpr int kHD = 64;
constexpr int kThreads = 512;  // WG0/WG1 gradient (query columns 0-63 / 64-127), WG2 dQ, warp 12 TMA, warp 13 MMA
constexpr int kTmaWarp = 12, kMmaWarp = 13;
// Register split (setmaxnreg): launched at 128 per thread (512 x 128 = 65536); the control warpgroup
// drops to 80 and the dQ warpgroup to 96 (freeing 4 x 32 x (48 + 32) = 10240), the gradient
// warpgroups rise to 168 (taking 2 x 4 x 32 x 40 = 10240).
constexpr int kRegsCtl = 80, kRegsDq = 96, kRegsGrad = 168;
static_assert(4 * 32 * (2 * kRegsGrad + kRegsDq + kRegsCtl) <= kThreads * 128, "register split exceeds the launch");
constexpr int kAtom = 128 * 128;   // one [128 rows x 64 bf16] swizzled atom
constexpr float kLog2e = 1.4426950408889634f;

// shared memory
constexpr int K_OFF = 0;                        // K tile (1 atom)
constexpr int V_OFF = K_OFF + kAtom;            // V tile
constexpr int kQStages = 3;  // Q / dO ring: the loads of tile i+2 overlap tile i (lse / delta come from L2)
constexpr int Q_OFF = V_OFF + kAtom;                   // kQStages stages
constexpr int DO_OFF = Q_OFF + kQStages * kAtom;       // kQStages stages
constexpr int DS_OFF = DO_OFF + kQStages * kAtom;      // dS^T, 2 buffers x 2 atoms (queries 0-63, 64-127)
constexpr int DQ_OFF = DS_OFF + 4 * kAtom;             // dQ staging: 2 boxes of [128 rows x 32 fp32], swizzled
constexpr int BAR_OFF = DQ_OFF + 2 * kAtom;
constexpr int SMEM = BAR_OFF + 256 + 1024;
static_assert(SMEM <= 232448, "shared memory budget");

// TMEM columns
constexpr int TM_S = 0, TM_DP = 128, TM_P = 256, TM_DV = 320, TM_DK = 384, TM_DQ = 448;

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

// TMA reduce-add of a shared-memory box into global fp32 (x, y non-negative, x * 4 bytes 16-aligned)
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
// AND of `v` over the dQ warpgroup (named barrier 1): every thread gets the same answer, so an error
// seen by one warp makes the whole group leave together instead of stranding the others at a barrier
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
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq,
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
  uint64_t* p_done = bars + 11;     // after (3) read P
  uint64_t* dq_full = bars + 12;
  uint64_t* dq_empty = bars + 13;
  uint64_t* acc_full = bars + 14;   // dK / dV of the item complete
  uint64_t* grad_done = bars + 15;  // [2]: per dS buffer, after (4)(5) of a tile read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = S / kT;
  const int n_items = T * BH;
  const int D = H * kHD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(&ld_full[i], 1);
      mbar_init(&ld_empty[i], 1 + 8);  // MMA commit + the 8 gradient warps (done with the tile)
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
    prefetch_tmap(&tm_qkv);
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
   if (warp == kTmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int ic = 0, lc = 0;
      bool ok = true;
      AST_DECL(a_pw);
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
        const Item it = item_of(i, BH, H);
        if (!(ok = mbar_wait(kv_empty, (ic & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
        mbar_arrive_expect_tx(kv_full, 2 * kAtom);
        const int krow = it.b * S + it.kb * kT;
        tma_load_2d(sK, &tm_qkv, kv_full, (H + it.h) * kHD, krow);
        tma_load_2d(sV, &tm_qkv, kv_full, (2 * H + it.h) * kHD, krow);
        for (int qi = it.kb; qi < T; ++qi, ++lc) {
          const int st = lc % kQStages;
          AST_T0(a_t);
          if (!(ok = mbar_wait(&ld_empty[st], ((lc / kQStages) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag))) break;
          AST_ADD(a_pw, a_t);
          mbar_arrive_expect_tx(&ld_full[st], 2 * kAtom);
          const int qrow = it.b * S + qi * kT;
          tma_load_2d(sQ + st * kAtom, &tm_qkv, &ld_full[st], it.h * kHD, qrow);
          tma_load_2d(sDO + st * kAtom, &tm_do, &ld_full[st], it.h * kHD, qrow);
        }
      }
      AST_FLUSH(11, a_pw);
    }
   } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_kk = make_idesc_bf16(128, 128, 0, 0);  // S^T, dP^T: both operands K-major
      constexpr uint32_t idesc_ts = make_idesc_bf16(128, kHD, 0, 1);  // dV: A TMEM, B MN-major
      constexpr uint32_t idesc_dk = make_idesc_bf16(128, kHD, 0, 1);  // dK: A K-major, B MN-major
      constexpr uint32_t idesc_dq = make_idesc_bf16(128, kHD, 1, 1);  // dQ: A M-major, B MN-major
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ), do_addr = smem_u32(sDO),
                     ds_addr = smem_u32(sDS);
      int ic = 0, lc = 0, tcount = 0;  // items, loaded tiles, tiles processed (phase counters)
      bool ok = true;
      AST_DECL(a_ld);
      AST_DECL(a_sf);
      AST_DECL(a_ds);
      AST_DECL(a_dq);
      AST_T0(a_loop);
      auto grad = [&](int v, int st, bool first) -> bool {  // MMAs (3)(4)(5) of the tile with counter v
        AST_T0(a_t1);
        if (!mbar_wait(ds_full, v & 1, err, kErrTimeoutTmemEmpty, abort_flag)) return false;
        AST_ADD(a_ds, a_t1);
        tc_fence_after();
        const uint64_t bdo = make_smem_desc(do_addr + st * kAtom, kAtom, 1024, 2);
        const uint64_t bq = make_smem_desc(q_addr + st * kAtom, kAtom, 1024, 2);
        const uint32_t dsb = ds_addr + (v & 1) * 2 * kAtom;
        const uint64_t ads = make_smem_desc(dsb, 16, 1024, 2);
#pragma unroll
        for (int k = 0; k < kT / 16; ++k) {  // (3) dV += P^T dO_i
          umma_bf16_ts(tmem + TM_DV, tmem + TM_P + k * 8, bdo + (k * 2048 >> 4), idesc_ts,
                       (!first || k > 0) ? 1u : 0u);
        }
        umma_commit(p_done);  // (3) has read P: the next tile's P may be written
#pragma unroll
        for (int k = 0; k < kT / 16; ++k) {  // (4) dK += dS^T Q_i
          const uint32_t off = (k >> 2) * kAtom + (k & 3) * 32;
          umma_bf16(tmem + TM_DK, ads + (off >> 4), bq + (k * 2048 >> 4), idesc_dk, (!first || k > 0) ? 1u : 0u);
        }
        AST_T0(a_t2);
        if (v > 0 && !mbar_wait(dq_empty, (v - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag)) return false;
        AST_ADD(a_dq, a_t2);
        tc_fence_after();
        const uint64_t adq = make_smem_desc(dsb, kAtom, 1024, 2);
        const uint64_t bk = make_smem_desc(k_addr, kAtom, 1024, 2);
#pragma unroll
        for (int k = 0; k < kT / 16; ++k)  // (5) dQ_i = dS K
          umma_bf16(tmem + TM_DQ, adq + (k * 2048 >> 4), bk + (k * 2048 >> 4), idesc_dq, k > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&grad_done[v & 1]);  // (4)(5) have read this tile's dS buffer
        umma_commit(&ld_empty[st]);
        return true;
      };
      for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
        const Item it = item_of(i, BH, H);
        if (!(ok = mbar_wait(kv_full, ic & 1, err, kErrTimeoutFull, abort_flag))) break;
        const uint64_t ak = make_smem_desc(k_addr, 16, 1024, 2), av = make_smem_desc(v_addr, 16, 1024, 2);
        int prev_st = 0;
        for (int qi = it.kb; qi < T && ok; ++qi, ++lc, ++tcount) {
          const int st = lc % kQStages;
          AST_T0(a_t3);
          if (!(ok = mbar_wait(&ld_full[st], (lc / kQStages) & 1, err, kErrTimeoutFull, abort_flag))) break;
          AST_ADD(a_ld, a_t3);
          AST_T0(a_t4);
          // S/dP may be overwritten once the gradient warpgroup has read the previous tile's
          if (tcount > 0 && !(ok = mbar_wait(s_free, (tcount - 1) & 1, err, kErrTimeoutTmemEmpty, abort_flag))) break;
          AST_ADD(a_sf, a_t4);
          tc_fence_after();
          const uint64_t bq = make_smem_desc(q_addr + st * kAtom, 16, 1024, 2);
          const uint64_t bdo = make_smem_desc(do_addr + st * kAtom, 16, 1024, 2);
#pragma unroll
          for (int k = 0; k < kHD / 16; ++k) {  // (1) S^T = K Q_i^T, (2) dP^T = V dO_i^T
            const uint64_t off = ((k & 3) * 32) >> 4;
            umma_bf16(tmem + TM_S, ak + off, bq + off, idesc_kk, k > 0 ? 1u : 0u);
            umma_bf16(tmem + TM_DP, av + off, bdo + off, idesc_kk, k > 0 ? 1u : 0u);
          }
          umma_commit(s_full);
          if (qi > it.kb && !(ok = grad(tcount - 1, prev_st, qi - 1 == it.kb))) break;
          prev_st = st;
        }
        if (!ok) break;
        if (!(ok = grad(tcount - 1, prev_st, T - 1 == it.kb))) break;
        umma_commit(acc_full);
        umma_commit(kv_empty);
      }
      AST_FLUSH(0, clock64() - a_loop);
      AST_FLUSH(1, a_ld);
      AST_FLUSH(2, a_sf);
      AST_FLUSH(3, a_ds);
      AST_FLUSH(4, a_dq);
      AST_FLUSH(13, tcount);
    }
   }
  } else if (warp < 8) {
    // ---------------- gradient warpgroups: thread = key row = TMEM lane; gw owns queries 64gw.. ----------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsGrad));
    const int gw = warp >> 2;
    const int r = threadIdx.x & 127;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float c = scale * kLog2e;
    int ic = 0, lc = 0, tcount = 0;
    bool ok = true;
    AST_DECL(g_w1);
    AST_DECL(g_w2);
    AST_DECL(g_w3);
    AST_T0(g_loop);
    for (int i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
      const Item it = item_of(i, BH, H);
      for (int qi = it.kb; qi < T; ++qi, ++lc, ++tcount) {
        const int st = lc % kQStages;
        AST_T0(g_t1);
        ok = mbar_wait(&ld_full[st], (lc / kQStages) & 1, err, kErrTimeoutFull, abort_flag) &&
             mbar_wait(s_full, tcount & 1, err, kErrTimeoutTmemFull, abort_flag);
        AST_ADD(g_w1, g_t1);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const float* sl = lse + (long long)it.bh * S + qi * kT;   // read through L1 / L2
        const float* sd = dvec + (long long)it.bh * S + qi * kT;
        {   // pull the next tile's lse / delta lines (this warpgroup's 64 queries: two 128-byte lines each)
            // into L1 now, so the next tile's quarter loads hit L1 instead of waiting on L2
          int nbh = it.bh, nq = qi + 1;
          if (nq >= T) {
            const int ni = snake_item(ic + 1);
            nbh = ni < n_items ? ni % BH : -1;
            nq = ni < n_items ? ni / BH : 0;
          }
          if (nbh >= 0 && (warp & 3) == 0 && lane < 4)
            prefetch_l1(((lane & 2) ? dvec : lse) + (long long)nbh * S + nq * kT + 64 * gw + 32 * (lane & 1));
        }
        const bool diag = qi == it.kb;
        uint8_t* ds_buf = sDS + (tcount & 1) * 2 * kAtom;
#pragma unroll 1
        for (int qt = 2 * gw; qt < 2 * gw + 2; ++qt) {  // 32 query columns at a time
          // this quarter's lse / delta first (32 values each, the same for every thread of the warpgroup,
          // so the loads hit L1 after the first warp), ahead of the TMEM loads they overlap
          float lv[32], dv[32];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(sl + qt * 32 + e);
            const float4 d4 = *reinterpret_cast<const float4*>(sd + qt * 32 + e);
            lv[e] = l4.x * kLog2e;
            lv[e + 1] = l4.y * kLog2e;
            lv[e + 2] = l4.z * kLog2e;
            lv[e + 3] = l4.w * kLog2e;
            dv[e] = d4.x;
            dv[e + 1] = d4.y;
            dv[e + 2] = d4.z;
            dv[e + 3] = d4.w;
          }
          uint32_t su[32], du[32];
          tmem_ld_32x32b_x32(lane_base + TM_S + qt * 32, su);
          tmem_ld_32x32b_x32(lane_base + TM_DP + qt * 32, du);
          tmem_ld_wait();
          if (qt == 2 * gw + 1) {  // this warpgroup's S/dP are in registers: the next tile's MMAs may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
          }
          if (qt == 2 * gw) {
            // P of the previous tile must have been read by its (3); this tile's dS buffer by (4)(5)
            // of the tile two back (each barrier is waited once per phase, in order)
            AST_T0(g_t2);
            if (tcount > 0) ok = mbar_wait(p_done, (tcount - 1) & 1, err, kErrTimeoutTmemFull, abort_flag);
            if (ok && tcount > 1)
              ok = mbar_wait(&grad_done[tcount & 1], ((tcount - 2) >> 1) & 1, err, kErrTimeoutTmemFull, abort_flag);
            AST_ADD(g_w2, g_t2);
            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
            tc_fence_after();
          }
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const int q = qt * 32 + e;  // query column
            float p[4], ds[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const bool vis = !diag || r <= q + u;
              p[u] = vis ? ex2_approx(fmaf(__uint_as_float(su[e + u]), c, -lv[e + u])) : 0.f;
              ds[u] = p[u] * (__uint_as_float(du[e + u]) - dv[e + u]);
            }
            pk[e >> 1] = pack_bf16x2(p[0], p[1]);
            pk[(e >> 1) + 1] = pack_bf16x2(p[2], p[3]);
            dk[e >> 1] = pack_bf16x2(ds[0], ds[1]);
            dk[(e >> 1) + 1] = pack_bf16x2(ds[2], ds[3]);
          }
          tmem_st_32x32b_x16(lane_base + TM_P + qt * 16, pk);
          // dS^T row r: queries 64*(qt/2).. live in atom qt/2; 16-byte chunk = 8 queries, swizzled by (r & 7)
          uint8_t* drow = ds_buf + (qt >> 1) * kAtom + r * 128;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int chunk = (qt & 1) * 4 + ch;
            *reinterpret_cast<uint4*>(drow + ((chunk ^ (r & 7)) << 4)) =
                make_uint4(dk[4 * ch], dk[4 * ch + 1], dk[4 * ch + 2], dk[4 * ch + 3]);
          }
        }
        if (!ok) break;
        tmem_st_wait();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(ds_full);
          mbar_arrive(&ld_empty[st]);  // the gradient warps are done with this stage's tile
        }
      }
      if (!ok) break;
      // ---- dK, dV of this key tile ----
      AST_T0(g_t3);
      ok = mbar_wait(acc_full, ic & 1, err, kErrTimeoutTmemFull, abort_flag);
      AST_ADD(g_w3, g_t3);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      // warpgroup 0 writes dK * scale (rotated back by -theta with a RoPE table), warpgroup 1 writes dV
      const long long row = (long long)it.b * S + it.kb * kT + r;
      __nv_bfloat16* dst = dqkv + row * ld_d + (gw == 0 ? D : 2 * D) + it.h * kHD;
      const float mul = gw == 0 ? scale : 1.f;
      const bool rot = gw == 0 && rope_cs != nullptr;
      const int pos = it.kb * kT + r;
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
            if (rot) {  // k was rotated by +theta in the forward: rotate its gradient by -theta
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
    if (threadIdx.x == 0) {
      AST_FLUSH(5, g_w1);
      AST_FLUSH(6, g_w2);
      AST_FLUSH(7, clock64() - g_loop);
      AST_FLUSH(12, g_w3);
    }
  } else if (warp < 12) {
    // ---------------- dQ warpgroup: thread = query row = TMEM lane ----------------
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsDq));
    const int r = threadIdx.x - 256;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    int tcount = 0;
    bool ok = true;
    AST_DECL(q_w1);
    AST_DECL(q_w2);
    AST_T0(q_loop);
    for (int ic = 0, i = snake_item(0); i < n_items && ok; i = snake_item(++ic)) {
      const Item it = item_of(i, BH, H);
      for (int qi = it.kb; qi < T; ++qi, ++tcount) {
        AST_T0(q_t1);
        ok = dq_wg_all(mbar_wait(dq_full, tcount & 1, err, kErrTimeoutTmemFull, abort_flag));
        AST_ADD(q_w1, q_t1);
        if (!ok) break;
        tc_fence_after();
        uint32_t qu[64];
        tmem_ld_32x32b_x32(lane_base + TM_DQ, *reinterpret_cast<uint32_t(*)[32]>(qu));
        tmem_ld_32x32b_x32(lane_base + TM_DQ + 32, *reinterpret_cast<uint32_t(*)[32]>(qu + 32));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        // stage dQ * scale in shared memory (two 128B-swizzled boxes of 32 columns), then one thread
        // adds both boxes into the fp32 accumulator with TMA reductions
        AST_T0(q_t2);
        if (r == 0) bulk_wait_read0();  // the previous tile's reductions have read the staging buffer
        dq_wg_sync();
        AST_ADD(q_w2, q_t2);
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          uint8_t* row = sDQ + bx * kAtom + r * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const int e = bx * 32 + ch * 4;
            *reinterpret_cast<float4*>(row + ((ch ^ (r & 7)) << 4)) =
                make_float4(__uint_as_float(qu[e]) * scale, __uint_as_float(qu[e + 1]) * scale,
                            __uint_as_float(qu[e + 2]) * scale, __uint_as_float(qu[e + 3]) * scale);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        dq_wg_sync();
        if (r == 0) {
          const int y = it.b * S + qi * kT;
          tma_reduce_add_2d(&tm_dq, sDQ, it.h * kHD, y);
          tma_reduce_add_2d(&tm_dq, sDQ + kAtom, it.h * kHD + 32, y);
          bulk_commit();
        }
      }
    }
    if (r == 0) bulk_wait0();  // every reduction has landed before the CTA exits
    if (r == 0) {
      AST_FLUSH(8, q_w1);
      AST_FLUSH(9, q_w2);
      AST_FLUSH(10, clock64() - q_loop);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

// delta[b*H + h][i] = sum_d dO[row, h, d] * O[row, h, d]: 8 lanes per (row, head), 16-byte loads;
// and zeroes the fp32 dQ accumulator (n4 float4s) in the same pass, which the backward kernel adds into
__global__ void bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                 long long ld_o, float* __restrict__ dvec, long long rows_h, int S, int H,
                                 float4* __restrict__ dq_zero, long long n4) {
  pdl_wait();
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
    dq_zero[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < rows_h * 8; t += stride) {
    const long long hr = t >> 3;
    const int part = (int)(t & 7);
    const long long row = hr / H;
    const int h = (int)(hr % H);
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * ld_o + h * kHD + part * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + row * ld_o + h * kHD + part * 8);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc += bf16_lo(av[k]) * bf16_lo(gv[k]) + bf16_hi(av[k]) * bf16_hi(gv[k]);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (part == 0) {
      const long long b = row / S;
      dvec[(b * H + h) * S + row % S] = acc;
    }
  }
}

// dqkv[:, 0:D] = bf16(dq_acc) (rotated by -theta with a RoPE table): 8 values per thread
__global__ void bwd_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv,
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

}  // namespace fab

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_fab() {
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

static bool encode_rows(PFN_cuTensorMapEncodeTiled_v12000 fn, CUtensorMap* tm, const void* base, long long cols,
                        long long rows, long long ld) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace pcb


// Same contract as pcb_attn_bwd_rope, on tcgen05: S % 128 == 0, HD 64 (this file) or 128
// (attention_bwd_tc128.cu), row strides % 8 == 0.
// Returns 0, -1 (unsupported shape), -5 (tensor-map encode) or -(1000 + cudaError) (launch).
// Copies the attention-backward cycle counters into out[16] and clears them; -1 when built without them.
int pcb_attn_bwd_stats(unsigned long long* out) {
#ifdef PCB_ATTN_STATS
  if (cudaMemcpyFromSymbol(out, pcb::fab::g_attn_stats, 16 * sizeof(unsigned long long)) != cudaSuccess) return -2;
  unsigned long long zero[16] = {};
  cudaMemcpyToSymbol(pcb::fab::g_attn_stats, zero, sizeof(zero));
  return 0;
#else
  (void)out;
  return -1;
#endif
}

int pcb_attn_bwd_tc128(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                       const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                       float scale, const float* rope_cs, int* err, cudaStream_t s);

int pcb_attn_bwd_tc(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                    const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                    int HD, float scale, const float* rope_cs, int* err, cudaStream_t s) {
  using namespace pcb;
  if (HD == 128)
    return pcb_attn_bwd_tc128(qkv, ld, out, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, scale, rope_cs, err, s);
  if (HD != 64 || S % 128 != 0 || ld % 8 || ld_o % 8 || ld_d % 8) return -1;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(lse) |
       reinterpret_cast<uintptr_t>(dvec) | reinterpret_cast<uintptr_t>(dq_acc)) & 15)
    return -1;
  auto fn = encode_fn_fab();
  if (!fn) return -5;
  CUtensorMap tq, td, tdq;
  if (!encode_rows(fn, &tq, qkv, 3LL * H * HD, (long long)B * S, ld) ||
      !encode_rows(fn, &td, dout, (long long)H * HD, (long long)B * S, ld_o))
    return -5;
  {  // fp32 dQ accumulator: boxes of 32 columns x 128 rows, 128-byte swizzle (the staging layout)
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(H) * HD, static_cast<cuuint64_t>(B) * S};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(H) * HD * 4};
    cuuint32_t box[2] = {32, 128};
    cuuint32_t es[2] = {1, 1};
    if (fn(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return -5;
  }
  const long long rows = (long long)B * S;
  step_launch(fab::bwd_delta_kernel, dim3(148 * 8), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(out),
             reinterpret_cast<const __nv_bfloat16*>(dout), ld_o, dvec, rows * H, S, H,
             reinterpret_cast<float4*>(dq_acc), rows * H * HD / 4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fab::attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fab::SMEM);
    attr = true;
  }
  static int num_sms = 0;
  if (num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (num_sms <= 0) num_sms = 148;
  }
  const int n_items = B * H * (S / fab::kT);
  const int grid = n_items < num_sms ? n_items : num_sms;  // persistent: one CTA per SM
  step_launch(fab::attn_bwd_tc_kernel, dim3(grid), dim3(fab::kThreads), fab::SMEM, s, tq, td, tdq, lse, dvec,
             reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d, S, H, scale, reinterpret_cast<const float2*>(rope_cs),
             B * H, err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return -(1000 + static_cast<int>(e));
  step_launch(fab::bwd_dq_convert_kernel, dim3(148 * 8), dim3(256), 0, s, dq_acc, reinterpret_cast<__nv_bfloat16*>(dqkv),
             ld_d, rows, H * HD, S, reinterpret_cast<const float2*>(rope_cs));
  const cudaError_t e2 = cudaGetLastError();
  return e2 == cudaSuccess ? 0 : -(1000 + static_cast<int>(e2));
}
