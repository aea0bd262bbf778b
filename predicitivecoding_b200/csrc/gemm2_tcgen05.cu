// tcgen05 GEMM on CTA pairs (cta_group::2): one 256 x BN output tile per 2-SM cluster.
//
// Each CTA of the pair loads its own half of the operands -- A rows [m0 + 128*rank, +128) and
// B columns [n0 + BN/2*rank, +BN/2) -- so per-SM operand traffic for a 128 x BN output slice is
// half of what the single-CTA kernel moves for B.  The leader CTA (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = BN; the accumulator rows of each CTA land in that
// CTA's own TMEM, so both CTAs run the same epilogue as the single-CTA kernel on 128 rows each.
//
// Synchronisation (all waits bounded):
//   full[s]   (leader)  armed by the leader's producer with both CTAs' bytes; both CTAs' TMA loads
//                       complete on it (cta_group::2 load form, leader barrier address)
//   empty[s]  (both)    released by the leader's MMA commit, multicast to both CTAs
//   tfull[a]  (both)    accumulator a ready: leader's commit multicast to both CTAs
//   tempty[a] (leader)  accumulator a drained: epilogue warps of both CTAs arrive (the peer remotely)
// No TMA load uses .multicast::cluster: each CTA fetches the tiles it stores.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm_epilogue.cuh"

namespace pcb {
namespace pair {

// Optional cycle counters (build with -DPCB_GEMM_STATS): where the roles of the pair kernel wait.
//   0 MMA issuer: cycles in its tile loop   1: waiting for a drained accumulator   2: waiting for operands
//   3 producer: waiting for a free stage    4 epilogue warp 2: waiting for an accumulator
//   5 epilogue warp 2: cycles draining      6 tiles issued by the MMA threads     7 producer cycles in its loop
//   8 epilogue warp 2: accumulator loads (coalesced path)   9: staging, operand loads and stores
#ifdef PCB_GEMM_STATS
__device__ unsigned long long g_pair_stats[12];
#define PAIR_STAT_DECL(v) long long v = 0
#define PAIR_STAT_T0(t) const long long t = clock64()
#define PAIR_STAT_ADD(v, t) v += clock64() - t
#define PAIR_STAT_FLUSH(i, v) atomicAdd(&g_pair_stats[i], (unsigned long long)(v))
#else
#define PAIR_STAT_DECL(v)
#define PAIR_STAT_T0(t)
#define PAIR_STAT_ADD(v, t)
#define PAIR_STAT_FLUSH(i, v)
#endif

constexpr int kBM = 128;  // rows per CTA (256 per pair)
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN, int EPI>
struct Cfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = (BN / 2) * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // per epilogue warp: 8 KB for the epilogues that stage two TMA boxes (bf16 output, SwiGLU, residual,
  // SwiGLU backward), 4 KB for the [32 x 32] fp32 transpose scratch of the coalesced path
  static constexpr bool kTwoBoxes =
      EPI == EPI_BF16 || EPI == EPI_SWIGLU || EPI == EPI_RESID_F32 || EPI == EPI_SWIGLU_BWD || EPI == EPI_GELU_BWD ||
      EPI == EPI_GELU;
  static constexpr int EPI_WARP_BYTES = kTwoBoxes ? 8192 : 4096;
  // the deepest operand ring that fits: 227 KB - 1 KB (barriers, alignment gap) - staging - 1 KB slack
  static constexpr int STAGES_FIT = (232448 - 2048 - 8 * EPI_WARP_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  // barriers in the first 256 bytes after the ring (then the auxiliary-tile barriers); the staging
  // area starts 1024-aligned for the 128-byte swizzle of the TMA boxes
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES + 1024;
  static constexpr int SMEM_BYTES = EPI_OFF + 8 * EPI_WARP_BYTES + 1024;
  static_assert(SMEM_BYTES <= 232448, "dynamic shared memory above the 227 KB per-block limit");
  static_assert(8 * (2 * STAGES + 4) + 8 <= 256, "barriers do not fit their 256-byte slot");
};

// Tile -> (split, row-pair block, column block).  Without a gather the row block varies fastest.
// With a fused all-gather the order is chunk-major, starting at this rank's own chunk and going
// round the ring, so the first wave computes on local rows while the other chunks are copied.
PCB_DEVICE void tile_coords(int tile, const GemmArgs& a, int num_m, int num_n, int& split, int& mb, int& nb) {
  split = tile % a.splits;
  const int rest = tile / a.splits;
  if (a.ag_world > 1) {
    const int mpc = a.ag_rows / (2 * kBM);
    const int tpc = mpc * num_n;
    const int c = (a.ag_rank + rest / tpc) % a.ag_world;
    const int r = rest % tpc;
    mb = c * mpc + r % mpc;
    nb = r / mpc;
  } else if (a.n_fastest) {
    nb = rest % num_n;
    mb = rest / num_n;
  } else {
    mb = rest % num_m;
    nb = rest / num_m;
  }
}

// Grouped GEMM: the expert of a 256-row tile and its k-block range; false when the tile is skipped
// (mode 1: past the rows in use; mode 2: an expert that received no rows).  The producer, the MMA
// issuer and the epilogue read the same segment table, so they skip the same tiles.
PCB_DEVICE bool grp_tile(const GemmArgs& a, int mb, int total_kb, int& e, int& kb0, int& kb1) {
  const int row0 = mb * 2 * kBM;
  if (a.grp_mode == 1) {
    if (row0 >= a.grp_seg[a.grp_count]) return false;
    int x = 0;
    while (x + 1 < a.grp_count && a.grp_seg[x + 1] <= row0) ++x;
    e = x;
    kb0 = 0;
    kb1 = total_kb;
    return true;
  }
  e = row0 / a.grp_m;
  kb0 = a.grp_seg[e] / kBK;
  kb1 = a.grp_seg[e + 1] / kBK;
  return kb1 > kb0;
}

PCB_DEVICE unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

PCB_DEVICE void red_release_gpu_add(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

PCB_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// bounded wait until *ctr >= target; false (and an error code) after the clock budget
PCB_DEVICE bool wait_counter(const unsigned int* ctr, unsigned int target, int* err, volatile int* abort_flag) {
  const long long t0 = clock64();
  while (ld_acquire_gpu(ctr) < target) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kSpinBudgetCycles) {
      record_error(err, kErrTimeoutChunk);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Epilogue warps of every CTA copy an equal share of each remote chunk of A into this rank's
// gathered buffer (16-byte loads from the peer over NVLink, local stores), then mark it done.
PCB_DEVICE void gather_chunks(const GemmArgs& a, int tid, int nthreads) {
  const long long chunk_vec = (long long)a.ag_rows * a.K / 8;   // uint4 per chunk
  const long long per = (chunk_vec + gridDim.x - 1) / gridDim.x;
  const long long v0 = blockIdx.x * per;
  const long long v1 = min(chunk_vec, v0 + per);
  for (int j = 1; j < a.ag_world; ++j) {
    const int c = (a.ag_rank + j) % a.ag_world;
    const uint4* src = reinterpret_cast<const uint4*>(a.ag_peers[c]) + c * chunk_vec;
    uint4* dst = reinterpret_cast<uint4*>(a.ag_local) + c * chunk_vec;
    // four independent 16-byte peer loads in flight per thread (NVLink latency is microseconds)
    for (long long v = v0 + tid; v < v1; v += 4LL * nthreads) {
      uint4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long idx = v + (long long)u * nthreads;
        if (idx < v1) a[u] = __ldcg(src + idx);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long idx = v + (long long)u * nthreads;
        if (idx < v1) dst[idx] = a[u];
      }
    }
    fence_proxy_async_global();
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
    if (tid == 0) {
      __threadfence();
      red_release_gpu_add(a.ag_ready + c, 1u);
    }
  }
}

// Epilogues that read an input tile of the output's shape (the residual stream; the SwiGLU
// pre-activations): with tensor maps, each warp loads its [32 x 32] input boxes by TMA into its
// staging buffer, finishes them in place and stores them by TMA.
template <int EPI>
PCB_DEVICE constexpr bool aux_tma() { return EPI == EPI_RESID_F32 || EPI == EPI_SWIGLU_BWD || EPI == EPI_GELU_BWD; }

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                     const GemmArgs args) {
  using C = Cfg<BN, EPI>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // two auxiliary-tile barriers per epilogue warp, 256 bytes into the 1 KB gap after the ring
  uint64_t* aux_bar = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (args.M + 2 * kBM - 1) / (2 * kBM);
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
      mbar_init(&tempty[s], 2 * kEpiWarps);
    }
    if (aux_tma<EPI>() && args.c_tma)
      for (int s = 0; s < 2 * kEpiWarps; ++s) mbar_init(aux_bar + s, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if ((EPI == EPI_BF16 || EPI == EPI_SWIGLU || EPI == EPI_GELU) && args.c_tma) prefetch_tmap(&tmC);
    if ((EPI == EPI_SWIGLU || EPI == EPI_GELU || aux_tma<EPI>()) && args.c_tma) prefetch_tmap(&tmD);
    if (aux_tma<EPI>() && args.c_tma) prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: everything above (barriers, tensor-map prefetch, TMEM) may overlap
  // the tail of the previous kernel in the stream; no global memory is touched before the previous
  // grid has completed and its writes are visible. The next kernel may be scheduled from here on (it
  // waits the same way before touching memory). Both are no-ops when the launch is not programmatic.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t ready_mask = args.ag_world > 1 ? (1u << args.ag_rank) : 0xffffffffu;
      PAIR_STAT_DECL(st_empty);
      PAIR_STAT_T0(st_loop);
      for (int tile = pair_id; tile < tiles && ok; tile += num_pairs) {
        int split, mb, nb;
        tile_coords(tile, args, num_m, num_n, split, mb, nb);
        int m0 = mb * 2 * kBM + rank * kBM;
        int n0 = nb * BN + rank * (BN / 2);
        int kb0 = split * args.kb_per_split;
        int kb1 = min(total_kb, kb0 + args.kb_per_split);
        int bk_off = 0;   // grouped, MN-major B: this expert's block along B's K coordinate
        if (args.grp_mode) {
          int e;
          if (!grp_tile(args, mb, total_kb, e, kb0, kb1)) continue;
          if (args.grp_mode == 1) {
            if (args.b_mn == 0) n0 += e * (int)args.grp_b_off;
            else bk_off = e * (int)args.grp_b_off;
          } else {
            m0 -= e * args.grp_m;   // A holds one expert's columns: local row coordinate
          }
        }
        if (args.ag_world > 1) {
          const int c = m0 / args.ag_rows;
          if (!((ready_mask >> c) & 1u)) {
            if (!wait_counter(args.ag_ready + c, gridDim.x, args.err, abort_flag)) { ok = false; break; }
            fence_proxy_async_global();
            ready_mask |= 1u << c;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          PAIR_STAT_T0(st_w);
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrTimeoutEmpty, abort_flag)) { ok = false; break; }
          PAIR_STAT_ADD(st_empty, st_w);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * kBK;
          if (args.a_mn == 0) {
            tma_load_2d_pair(sa, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int p = 0; p < kBM / 64; ++p) tma_load_2d_pair(sa + p * 8192, &tmA, &full[stage], m0 + 64 * p, k0);
          }
          if (args.b_mn == 0) {
            tma_load_2d_pair(sb, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int p = 0; p < BN / 128; ++p)
              tma_load_2d_pair(sb + p * 8192, &tmB, &full[stage], n0 + 64 * p, k0 + bk_off);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      PAIR_STAT_FLUSH(3, st_empty);
      PAIR_STAT_FLUSH(7, clock64() - st_loop);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader only) ----------------
      const uint32_t idesc = make_idesc_bf16(2 * kBM, BN, args.a_mn, args.b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      PAIR_STAT_DECL(st_tempty);
      PAIR_STAT_DECL(st_full);
      PAIR_STAT_DECL(st_tiles);
      PAIR_STAT_T0(st_loop);
      for (int tile = pair_id; tile < tiles && ok; tile += num_pairs) {
        const int split = tile % args.splits;   // same in both tile orders
        int kb0 = split * args.kb_per_split;
        int kb1 = min(total_kb, kb0 + args.kb_per_split);
        if (args.grp_mode) {
          int sp, mb, nb, e;
          tile_coords(tile, args, num_m, num_n, sp, mb, nb);
          if (!grp_tile(args, mb, total_kb, e, kb0, kb1)) continue;
        }
        PAIR_STAT_T0(st_w0);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.err, kErrTimeoutTmemEmpty, abort_flag)) { ok = false; break; }
        PAIR_STAT_ADD(st_tempty, st_w0);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          PAIR_STAT_T0(st_w1);
          if (!mbar_wait(&full[stage], phase, args.err, kErrTimeoutFull, abort_flag)) { ok = false; break; }
          PAIR_STAT_ADD(st_full, st_w1);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = args.a_mn ? make_smem_desc(sa + k * 2048, 8192, 1024, 2)
                                          : make_smem_desc(sa + k * 32, 16, 1024, 2);
            const uint64_t bd = args.b_mn ? make_smem_desc(sb + k * 2048, 8192, 1024, 2)
                                          : make_smem_desc(sb + k * 32, 16, 1024, 2);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
#ifdef PCB_GEMM_STATS
        ++st_tiles;
#endif
      }
      PAIR_STAT_FLUSH(0, clock64() - st_loop);
      PAIR_STAT_FLUSH(1, st_tempty);
      PAIR_STAT_FLUSH(2, st_full);
      PAIR_STAT_FLUSH(6, st_tiles);
    }
  } else {
    // ---------------- epilogue warps (both CTAs, 128 rows each) ----------------
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty[1]), 0);
    if (args.ag_world > 1) gather_chunks(args, threadIdx.x - 64, 32 * kEpiWarps);
    int acc = 0;
    uint32_t acc_phase = 0;
    PAIR_STAT_DECL(st_tfull);
    PAIR_STAT_DECL(st_body);
    uint8_t* aux_stage = smem + C::EPI_OFF + (warp - 2) * C::EPI_WARP_BYTES;
    uint32_t aux_ph = 0u;   // bit b: parity of buffer b's next completion
    int store_box = 0;      // bf16 TMA-store path: the staging box used next (alternates across tiles too)
    bool aux_ok = true;
    for (int tile = pair_id; tile < tiles && aux_ok; tile += num_pairs) {
      int split_unused, mb, nb;
      tile_coords(tile, args, num_m, num_n, split_unused, mb, nb);
      long long boff = 0;   // grouped, mode 1: this expert's bias block
      if (args.grp_mode) {
        int e, g0, g1;
        if (!grp_tile(args, mb, total_kb, e, g0, g1)) continue;
        if (args.grp_mode == 1) boff = (long long)e * args.grp_bias_off;
      }
      const int m = mb * 2 * kBM + rank * kBM + row;
      const int n0 = nb * BN;
      const bool row_ok = m < args.M;
      const int row0_aux = mb * 2 * kBM + rank * kBM + q * 32;
      // input boxes of chunk i (accumulator columns [32 (half + 2 i), +32)) into buffer buf
      auto aux_request = [&](int i, int buf) {
        uint64_t* bar = &aux_bar[(warp - 2) * 2 + buf];
        uint8_t* box = aux_stage + buf * 4096;
        const int n = n0 + (half + 2 * i) * 32;
        mbar_arrive_expect_tx(bar, EPI == EPI_GELU_BWD ? 2048 : 4096);
        if (EPI == EPI_RESID_F32 || EPI == EPI_GELU_BWD) {
          tma_load_2d(box, &tmD, bar, n, row0_aux);
        } else {
          const int gx = (n >> 6) * 128 + (n & 63);
          tma_load_2d(box, &tmD, bar, gx, row0_aux);
          tma_load_2d(box + 2048, &tmD, bar, gx + 64, row0_aux);
        }
      };
      if (aux_tma<EPI>() && args.c_tma && lane == 0) {
        bulk_group_wait_read<0>();   // the previous tile's stores have read both buffers
        aux_request(0, 0);
        if (BN / 64 > 1) aux_request(1, 1);
      }
      PAIR_STAT_T0(st_w2);
      if (!mbar_wait(&tfull[acc], acc_phase, args.err, kErrTimeoutTmemFull, abort_flag)) break;
      PAIR_STAT_ADD(st_tfull, st_w2);
      PAIR_STAT_T0(st_b);
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (aux_tma<EPI>() && args.c_tma) {
        // chunk i of this warp = accumulator columns [32 (half + 2 i), +32); input boxes of chunk i go
        // to buffer i & 1 (4 KB: one fp32 box, or the gate and up bf16 boxes of 2 KB); the boxes of
        // chunks 0 and 1 were requested before the accumulator wait, chunk i + 2 is requested as soon as
        // the store of chunk i has read buffer i & 1
        constexpr int NCH = BN / 64;
#pragma unroll 1
        for (int i = 0; i < NCH; ++i) {
          const int c = half + 2 * i;
          const int buf = i & 1;
          uint8_t* box = aux_stage + buf * 4096;
          float v[32];
          tmem_load_f32x32(tbase + c * 32, v);
          const bool got = mbar_wait(&aux_bar[(warp - 2) * 2 + buf], (aux_ph >> buf) & 1u, args.err, kErrTimeoutAux,
                                     abort_flag);
          if (!__all_sync(0xffffffffu, got)) {   // the warp leaves together
            aux_ok = false;
            break;
          }
          aux_ph ^= 1u << buf;
          const int n = n0 + c * 32;
          if (EPI == EPI_RESID_F32) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4* cell = reinterpret_cast<float4*>(box + lane * 128 + ((j ^ (lane & 7)) << 4));
              float4 a = *cell;
              float o[4] = {v[4 * j] * args.alpha, v[4 * j + 1] * args.alpha, v[4 * j + 2] * args.alpha,
                            v[4 * j + 3] * args.alpha};
              if (args.bias != nullptr) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int col = n + 4 * j + e;
                  if (col < args.N)
                    o[e] += args.bias_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(args.bias)[col])
                                           : reinterpret_cast<const float*>(args.bias)[col];
                }
              }
              a.x += o[0];
              a.y += o[1];
              a.z += o[2];
              a.w += o[3];
              *cell = a;
            }
          } else if (EPI == EPI_GELU_BWD) {  // pre box [32 rows x 32] bf16, 64-byte rows, 64-byte swizzle
            const int sw = (lane >> 1) & 3;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              uint4* pp = reinterpret_cast<uint4*>(box + lane * 64 + ((cc ^ sw) << 4));
              const uint4 p4 = *pp;
              const uint32_t pw[4] = {p4.x, p4.y, p4.z, p4.w};
              uint32_t ow[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                ow[k] = pack_bf16x2(args.alpha * v[8 * cc + 2 * k] * gelu_tanh_grad_fast(bf16_lo(pw[k])),
                                    args.alpha * v[8 * cc + 2 * k + 1] * gelu_tanh_grad_fast(bf16_hi(pw[k])));
              *pp = make_uint4(ow[0], ow[1], ow[2], ow[3]);
            }
          } else {  // EPI_SWIGLU_BWD: gate box at box, up box at box + 2048 (64-byte rows, 64-byte swizzle)
            const int sw = (lane >> 1) & 3;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              uint4* gp = reinterpret_cast<uint4*>(box + lane * 64 + ((cc ^ sw) << 4));
              uint4* up = reinterpret_cast<uint4*>(box + 2048 + lane * 64 + ((cc ^ sw) << 4));
              const uint4 g4 = *gp, u4 = *up;
              const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
              const uint32_t uw[4] = {u4.x, u4.y, u4.z, u4.w};
              uint32_t dgw[4], duw[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                float dgv[2], duv[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const float g = e ? bf16_hi(gw[k]) : bf16_lo(gw[k]);
                  const float u = e ? bf16_hi(uw[k]) : bf16_lo(uw[k]);
                  const float dh = args.alpha * v[8 * cc + 2 * k + e];
                  const float sg = __fdividef(1.f, 1.f + __expf(-g));
                  duv[e] = dh * g * sg;
                  dgv[e] = dh * u * sg * (1.f + g * (1.f - sg));
                }
                dgw[k] = pack_bf16x2(dgv[0], dgv[1]);
                duw[k] = pack_bf16x2(duv[0], duv[1]);
              }
              *gp = make_uint4(dgw[0], dgw[1], dgw[2], dgw[3]);
              *up = make_uint4(duw[0], duw[1], duw[2], duw[3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (EPI == EPI_RESID_F32 || EPI == EPI_GELU_BWD) {
              tma_store_2d(&tmC, box, n, row0_aux);
            } else {
              const int gx = (n >> 6) * 128 + (n & 63);
              tma_store_2d(&tmC, box, gx, row0_aux);
              tma_store_2d(&tmC, box + 2048, gx + 64, row0_aux);
            }
            bulk_group_commit();
            if (i + 2 < NCH) {
              bulk_group_wait_read<0>();
              aux_request(i + 2, buf);
            }
          }
        }
      } else if (EPI == EPI_GELU && args.c_tma) {
        // per 32-column chunk: pre = alpha acc + bias and act = gelu(bf16(pre)), staged as two [32 x 32]
        // bf16 boxes (64-byte rows, 64-byte swizzle: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)) and
        // written by TMA stores into C and D; the two box pairs of the staging area alternate
        uint8_t* stg = smem + C::EPI_OFF + (warp - 2) * C::EPI_WARP_BYTES;
        const int row0 = mb * 2 * kBM + rank * kBM + q * 32;
        const int sw = (lane >> 1) & 3;
#pragma unroll 1
        for (int i = 0; i < BN / 64; ++i) {
          const int c = half + 2 * i;
          const int n = n0 + c * 32;
          float v[32], bv[32];
          tmem_load_f32x32(tbase + c * 32, v);
          if (args.bias != nullptr) {
            const int nvalid = min(32, args.N - n);
            if (args.bias_bf16) load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(args.bias) + boff + n, bv, nvalid);
            else load_f32x32(reinterpret_cast<const float*>(args.bias) + boff + n, bv, nvalid);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) bv[j] = 0.f;
          }
          uint32_t pp[16], pa[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            pp[j] = pack_bf16x2(fmaf(v[2 * j], args.alpha, bv[2 * j]), fmaf(v[2 * j + 1], args.alpha, bv[2 * j + 1]));
            pa[j] = pack_bf16x2(gelu_tanh_fast(bf16_lo(pp[j])), gelu_tanh_fast(bf16_hi(pp[j])));
          }
          uint8_t* box = stg + store_box * 4096;
          if (lane == 0) bulk_group_wait_read<1>();   // the stores that last read this box pair are done
          __syncwarp();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int off = lane * 64 + ((cc ^ sw) << 4);
            *reinterpret_cast<uint4*>(box + off) = make_uint4(pp[4 * cc], pp[4 * cc + 1], pp[4 * cc + 2], pp[4 * cc + 3]);
            *reinterpret_cast<uint4*>(box + 2048 + off) =
                make_uint4(pa[4 * cc], pa[4 * cc + 1], pa[4 * cc + 2], pa[4 * cc + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, box, n, row0);
            tma_store_2d(&tmD, box + 2048, n, row0);
            bulk_group_commit();
          }
          store_box ^= 1;
        }
      } else if (EPI == EPI_SWIGLU && args.c_tma) {
        // per 128-column group: this warp's 32 gate and 32 up columns of pre and the 32 act columns
        // they make, each staged as a [32 x 32] bf16 box (64-byte rows, 64-byte swizzle: 16-byte
        // chunk c of row r at c ^ ((r >> 1) & 3)) and written by TMA stores
        uint8_t* stg = smem + C::EPI_OFF + (warp - 2) * C::EPI_WARP_BYTES;
        const int row0 = mb * 2 * kBM + rank * kBM + q * 32;
#pragma unroll 1
        for (int g = 0; g < BN / 128; ++g) {
          const int h = half;
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tbase + g * 128 + h * 32, rg);
          tmem_ld_32x32b_x32(tbase + g * 128 + 64 + h * 32, ru);
          tmem_ld_wait();
          uint32_t pg[16], pu[16], pa[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float g0 = __uint_as_float(rg[2 * j]) * args.alpha, g1 = __uint_as_float(rg[2 * j + 1]) * args.alpha;
            const float u0 = __uint_as_float(ru[2 * j]) * args.alpha, u1 = __uint_as_float(ru[2 * j + 1]) * args.alpha;
            pg[j] = pack_bf16x2(g0, g1);
            pu[j] = pack_bf16x2(u0, u1);
            const float gb0 = bf16_lo(pg[j]), gb1 = bf16_hi(pg[j]);
            const float ub0 = bf16_lo(pu[j]), ub1 = bf16_hi(pu[j]);
            pa[j] = pack_bf16x2(__fdividef(gb0, 1.f + __expf(-gb0)) * ub0, __fdividef(gb1, 1.f + __expf(-gb1)) * ub1);
          }
          if (lane == 0) bulk_group_wait_read<0>();   // the previous group's stores have read the boxes
          __syncwarp();
          const int sw = (lane >> 1) & 3;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int off = lane * 64 + ((c ^ sw) << 4);
            *reinterpret_cast<uint4*>(stg + off) = make_uint4(pg[4 * c], pg[4 * c + 1], pg[4 * c + 2], pg[4 * c + 3]);
            *reinterpret_cast<uint4*>(stg + 2048 + off) = make_uint4(pu[4 * c], pu[4 * c + 1], pu[4 * c + 2], pu[4 * c + 3]);
            *reinterpret_cast<uint4*>(stg + 4096 + off) = make_uint4(pa[4 * c], pa[4 * c + 1], pa[4 * c + 2], pa[4 * c + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stg, n0 + g * 128 + h * 32, row0);
            tma_store_2d(&tmC, stg + 2048, n0 + g * 128 + 64 + h * 32, row0);
            tma_store_2d(&tmD, stg + 4096, (n0 >> 1) + g * 64 + h * 32, row0);
            bulk_group_commit();
          }
        }
      } else if (EPI == EPI_SWIGLU) {
#pragma unroll 1
        for (int g = 0; g < BN / 128; ++g) {
          const int h = half;
          float gv[32], uv[32];
          tmem_load_f32x32(tbase + g * 128 + h * 32, gv);
          tmem_load_f32x32(tbase + g * 128 + 64 + h * 32, uv);
          const int ncol = n0 + g * 128 + h * 32;
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
              const float gg = __bfloat162float(__float2bfloat16_rn(gv[j]));
              const float uu = __bfloat162float(__float2bfloat16_rn(uv[j]));
              o[j] = __fdividef(gg, 1.f + __expf(-gg)) * uu;
            }
            const int fcol = (n0 >> 1) + g * 64 + h * 32;
            store_bf16x32(reinterpret_cast<__nv_bfloat16*>(args.D) + (long long)m * args.ldd + fcol, o, nvalid);
          }
        }
      } else if (EPI == EPI_BF16 && args.c_tma) {
        // 64-column blocks: two accumulator chunks -> alpha, bias, RoPE -> bf16 row of 128 bytes per
        // lane, staged in the 128-byte-swizzled layout of a [32 x 64] box and written by one TMA store.
        // The two boxes of a warp alternate over all of its blocks, across tiles too (with BN = 128 a
        // tile has one block per warp); before a box is rewritten every store but the latest, which
        // read the other box, has finished reading.
        uint8_t* stg = smem + C::EPI_OFF + (warp - 2) * C::EPI_WARP_BYTES;
        const int row0 = mb * 2 * kBM + rank * kBM + q * 32;
#pragma unroll 1
        for (int c2 = half; c2 < BN / 64; c2 += 2) {
          const int bx = store_box;
          store_box ^= 1;
          float v[64];
          {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tbase + c2 * 64, r0);
            tmem_ld_32x32b_x32(tbase + c2 * 64 + 32, r1);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              v[j] = __uint_as_float(r0[j]);
              v[32 + j] = __uint_as_float(r1[j]);
            }
          }
          const int nb0 = n0 + c2 * 64;
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] *= args.alpha;
          if (args.bias != nullptr) {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const int n = nb0 + j;
              if (n < args.N)
                v[j] += args.bias_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(args.bias)[n])
                                       : reinterpret_cast<const float*>(args.bias)[n];
            }
          }
          if (args.rope_cs != nullptr && nb0 < args.rope_cols && row_ok) {
            const float2* cs = reinterpret_cast<const float2*>(args.rope_cs) + (long long)(m % args.rope_S) * (args.rope_hd >> 1);
#pragma unroll
            for (int j = 0; j < 64; j += 2) {
              const int n = nb0 + j;
              if (n < args.rope_cols) {
                const float2 cv = cs[(n % args.rope_hd) >> 1];
                const float x0 = v[j], x1 = v[j + 1];
                v[j] = x0 * cv.x - x1 * cv.y;
                v[j + 1] = x0 * cv.y + x1 * cv.x;
              }
            }
          }
          uint8_t* box = stg + bx * 4096;
          if (lane == 0) bulk_group_wait_read<1>();   // the store that last read this box is done with it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(box + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, box, nb0, row0);
            bulk_group_commit();
          }
        }
      } else if (epi_coalesced<EPI>()) {
        // transpose each 32x32 chunk through this warp's shared scratch (16-byte cells, XOR-swizzled by
        // row) so that 8 lanes then cover one 128-byte row segment of the output
        float4* scr = reinterpret_cast<float4*>(smem + C::EPI_OFF + (warp - 2) * C::EPI_WARP_BYTES);
        const int row0 = mb * 2 * kBM + rank * kBM + q * 32;
        float sq = 0.f;
        PAIR_STAT_DECL(st_ld);
        PAIR_STAT_DECL(st_st);
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          PAIR_STAT_T0(st_l0);
          tmem_load_f32x32(tbase + c * 32, v);
          PAIR_STAT_ADD(st_ld, st_l0);
          PAIR_STAT_T0(st_s0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            scr[lane * 8 + (j ^ (lane & 7))] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          __syncwarp();
          const int c4 = lane & 7, ncol = n0 + c * 32 + c4 * 4;
          float pf[8][8];
#pragma unroll
          for (int it = 0; it < 8; ++it) {   // every row's operand loads in flight first
            const int rr = it * 4 + (lane >> 3);
            epi_prefetch<EPI>(args, row0 + rr, ncol, pf[it], row0 + rr < args.M);
          }
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            const float4 x = scr[rr * 8 + (c4 ^ (rr & 7))];
            float e[4] = {x.x, x.y, x.z, x.w};
            sq += epilogue_vec4<EPI>(args, row0 + rr, ncol, e, pf[it], row0 + rr < args.M, boff);
          }
          __syncwarp();
          PAIR_STAT_ADD(st_st, st_s0);
        }
        if (warp == 2 && lane == 0) {
          PAIR_STAT_FLUSH(8, st_ld);
          PAIR_STAT_FLUSH(9, st_st);
        }
        if (EPI == EPI_PC_PRED && args.pc_energy != nullptr) {
          sq = warp_sum(sq);
          if (lane == 0) atomicAdd(args.pc_energy, sq);
        }
      } else if (EPI == EPI_SWIGLU_BWD) {
        // row path with the next chunk's gate / up rows prefetched while this chunk is finished
        const __nv_bfloat16* pre = reinterpret_cast<const __nv_bfloat16*>(args.aux) + (long long)m * args.ldaux;
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.C) + (long long)m * args.ldc;
        auto gcol_of = [&](int c) -> long long {
          const int n = n0 + c * 32;
          return (long long)(n >> 6) * 128 + (n & 63);
        };
        const bool vec_ok = (args.ldaux % 8) == 0 && (args.ldc % 8) == 0 &&
                            ((reinterpret_cast<uintptr_t>(args.aux) | reinterpret_cast<uintptr_t>(args.C)) & 15) == 0;
        auto fetch = [&](int c, uint4 (&g4)[4], uint4 (&u4)[4]) {
          const int nvalid = min(32, args.N - (n0 + c * 32));
          if (vec_ok && row_ok && nvalid >= 32) {
            const uint4* gp = reinterpret_cast<const uint4*>(pre + gcol_of(c));
            const uint4* up = reinterpret_cast<const uint4*>(pre + gcol_of(c) + 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              g4[j] = gp[j];
              u4[j] = up[j];
            }
          }
        };
        uint4 cg[4], cu[4], ng[4], nu[4];
        fetch(half, cg, cu);
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          if (c + 2 < BN / 32) fetch(c + 2, ng, nu);
          float v[32];
          tmem_load_f32x32(tbase + c * 32, v);
          const int n = n0 + c * 32;
          const int nvalid = min(32, args.N - n);
          if (vec_ok && row_ok && nvalid >= 32) {
            float dg[32], du[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t gw = reinterpret_cast<const uint32_t*>(cg)[j >> 1];
              const uint32_t uw = reinterpret_cast<const uint32_t*>(cu)[j >> 1];
              const float g = (j & 1) ? bf16_hi(gw) : bf16_lo(gw);
              const float u = (j & 1) ? bf16_hi(uw) : bf16_lo(uw);
              const float dh = args.alpha * v[j];
              const float sg = __fdividef(1.f, 1.f + __expf(-g));
              du[j] = dh * g * sg;
              dg[j] = dh * u * sg * (1.f + g * (1.f - sg));
            }
            store_bf16x32(out + gcol_of(c), dg, 32);
            store_bf16x32(out + gcol_of(c) + 64, du, 32);
          } else {
            epilogue_chunk<EPI>(args, m, n, v, row_ok, boff);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            cg[j] = ng[j];
            cu[j] = nu[j];
          }
        }
      } else {
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          tmem_load_f32x32(tbase + c * 32, v);
          epilogue_chunk<EPI>(args, m, n0 + c * 32, v, row_ok, boff);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty[acc]);
        else mbar_arrive_remote(acc ? tempty_leader1 : tempty_leader0);
      }
      PAIR_STAT_ADD(st_body, st_b);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (warp == 2 && lane == 0) {
      PAIR_STAT_FLUSH(4, st_tfull);
      PAIR_STAT_FLUSH(5, st_body);
    }
  }

  if ((EPI == EPI_BF16 || EPI == EPI_SWIGLU || EPI == EPI_GELU || aux_tma<EPI>()) && args.c_tma && warp >= 2 &&
      lane == 0)
    bulk_group_wait_all();  // every TMA store has landed before the CTA exits
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // both CTAs done with TMEM and with each other's barriers
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace pair

// Copies the pair-kernel cycle counters into out[12] and clears them; -1 when built without them.
int pcb_gemm_pair_stats(unsigned long long* out) {
#ifdef PCB_GEMM_STATS
  if (cudaMemcpyFromSymbol(out, pair::g_pair_stats, 12 * sizeof(unsigned long long)) != cudaSuccess) return -2;
  unsigned long long zero[12] = {};
  cudaMemcpyToSymbol(pair::g_pair_stats, zero, sizeof(zero));
  return 0;
#else
  (void)out;
  return -1;
#endif
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn2() {
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

static bool make_map2(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                      uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B, bool f32 = false) {
  auto fn = encode_fn2();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
            dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Programmatic dependent launch of the pair kernel (PCB_PDL=0 turns it off).
static bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("PCB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int BN, int EPI>
static int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& td,
                       const GemmArgs& a, int grid, cudaStream_t s) {
  using C = pair::Cfg<BN, EPI>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(pair::gemm_pair_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(pair::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  if (a.ag_world > 1) {
    // with a fused gather, CTAs wait on each other's copies: all of them must be resident at once
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
  } else {
    // the prologue may overlap the previous kernel's tail (the kernel waits before touching memory)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, pair::gemm_pair_kernel<BN, EPI>, ta, tb, tc, td, a);
  if (e != cudaSuccess && a.ag_world > 1) {
    // cooperative + cluster refused: one CTA per SM with grid <= SM count is resident anyway on a
    // stream of its own; the chunk waits stay bounded either way
    cudaGetLastError();
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, pair::gemm_pair_kernel<BN, EPI>, ta, tb, tc, td, a);
  }
  return e == cudaSuccess ? 0 : -3;
}

template <int BN>
static int dispatch_pair(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                         const CUtensorMap& td, const GemmArgs& a, int grid, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: return launch_pair<BN, EPI_BF16>(ta, tb, tc, td, a, grid, s);
    case EPI_F32: return launch_pair<BN, EPI_F32>(ta, tb, tc, td, a, grid, s);
    case EPI_ACC_F32: return launch_pair<BN, EPI_ACC_F32>(ta, tb, tc, td, a, grid, s);
    case EPI_RED_F32: return launch_pair<BN, EPI_RED_F32>(ta, tb, tc, td, a, grid, s);
    case EPI_GELU: return launch_pair<BN, EPI_GELU>(ta, tb, tc, td, a, grid, s);
    case EPI_SWIGLU: return launch_pair<BN, EPI_SWIGLU>(ta, tb, tc, td, a, grid, s);
    case EPI_SWIGLU_BWD: return launch_pair<BN, EPI_SWIGLU_BWD>(ta, tb, tc, td, a, grid, s);
    case EPI_GELU_BWD: return launch_pair<BN, EPI_GELU_BWD>(ta, tb, tc, td, a, grid, s);
    case EPI_PC_PRED: return launch_pair<BN, EPI_PC_PRED>(ta, tb, tc, td, a, grid, s);
    case EPI_PC_STATE: return launch_pair<BN, EPI_PC_STATE>(ta, tb, tc, td, a, grid, s);
    case EPI_PC_WUPD: return launch_pair<BN, EPI_PC_WUPD>(ta, tb, tc, td, a, grid, s);
    case EPI_BF16_ACC: return launch_pair<BN, EPI_BF16_ACC>(ta, tb, tc, td, a, grid, s);
    case EPI_RESID_F32: return launch_pair<BN, EPI_RESID_F32>(ta, tb, tc, td, a, grid, s);
    case EPI_RS_BF16: return launch_pair<BN, EPI_RS_BF16>(ta, tb, tc, td, a, grid, s);
    default: return -2;
  }
}

}  // namespace pcb

using namespace pcb;

// CTA-pair GEMM launcher: same contract as pcb_gemm_launch.  bn in {128, 256}; splits >= 1 (split-K only
// with EPI_RED_F32).  Returns 0 on success.
int pcb_gemm_pair_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, int epi,
                         GemmArgs args, int bn, int splits, int num_sms, cudaStream_t stream) {
  const int M = args.M, N = args.N, K = args.K;
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  if ((lda % 8) != 0 || (ldb % 8) != 0) return -1;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15)) return -1;
  if (bn != 128 && bn != 256) return -1;
  if (num_sms <= 0) num_sms = 148;
  args.a_mn = a_mn;
  args.b_mn = b_mn;
  const int num_m = (M + 255) / 256;
  const int num_n = (N + bn - 1) / bn;
  const int total_kb = (K + 63) / 64;
  if (splits < 1) splits = 1;
  if (splits > 1 && epi != EPI_RED_F32) return -4;
  if (args.ag_world > 1) {
    // fused gather: K-major A spanning all chunks, whole 256-row tiles per chunk, no split-K
    if (a_mn != 0 || lda != K || (K % 8) != 0 || args.ag_rows % 256 != 0 || args.ag_world > 32 ||
        (long long)args.ag_rows * args.ag_world != M || splits != 1 || args.ag_peers == nullptr ||
        args.ag_ready == nullptr || args.ag_local != A)
      return -6;
  }
  if (epi == EPI_RS_BF16 && (args.rs_peers == nullptr || args.rs_rows <= 0 || (M % args.rs_rows) != 0)) return -6;
  int kbps = (total_kb + splits - 1) / splits;
  splits = (total_kb + kbps - 1) / kbps;
  args.splits = splits;
  args.kb_per_split = kbps;
  // grouped GEMM: A of a weight gradient holds one expert's columns (grp_m); B of the rows mode
  // stacks grp_count expert blocks
  const long long a_rows = args.grp_mode == 2 ? args.grp_m : M;
  const long long b_ext = (args.grp_mode == 1 ? args.grp_count : 1) * (long long)(b_mn ? K : N);
  CUtensorMap ta, tb;
  bool ok = a_mn == 0 ? make_map2(&ta, A, K, a_rows, lda, 64, 128) : make_map2(&ta, A, a_rows, K, lda, 64, 64);
  if (!ok) return -5;
  ok = b_mn == 0 ? make_map2(&tb, B, K, b_ext, ldb, 64, bn / 2) : make_map2(&tb, B, N, b_ext, ldb, 64, 64);
  if (!ok) return -5;
  // Tile order: the pairs running at once should share the operand with the larger footprint, so that
  // it crosses from DRAM once per wave. With A larger (M > N) the column blocks of one row block run
  // side by side; otherwise the row blocks of one column block do. PCB_GEMM_RASTER=1 / 2 forces
  // row-fastest / column-fastest (measurement).
  static const int raster_env = [] {
    const char* e = getenv("PCB_GEMM_RASTER");
    return e ? atoi(e) : 0;
  }();
  args.n_fastest = raster_env == 1 ? 0 : raster_env == 2 ? 1 : (M > N ? 1 : 0);
  // bf16 output through TMA stores when C can be described by a tensor map (16-byte aligned base and
  // row stride); [32 x 64] boxes, clipped by the hardware at the M / N edges
  CUtensorMap tc, td;
  memset(&tc, 0, sizeof(tc));
  memset(&td, 0, sizeof(td));
  args.c_tma = 0;
  const bool c_ok = (reinterpret_cast<uintptr_t>(args.C) & 15) == 0 && (args.ldc % 8) == 0;
  if (epi == EPI_BF16 && c_ok && make_map2(&tc, args.C, N, M, args.ldc, 64, 32)) args.c_tma = 1;
  // SwiGLU forward: pre (C, [M, N]) and act (D, [M, N / 2]) in [32 x 32] boxes with 64-byte swizzle
  if (epi == EPI_SWIGLU && c_ok && args.D != nullptr && (reinterpret_cast<uintptr_t>(args.D) & 15) == 0 &&
      (args.ldd % 8) == 0 && make_map2(&tc, args.C, N, M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_map2(&td, args.D, N / 2, M, args.ldd, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    args.c_tma = 1;
  // residual add (fp32 x_out = x_in + f(x)) and SwiGLU backward (bf16 pre in, bf16 d(pre) out): the
  // input tile is loaded by TMA through the D map slot, the output stored by TMA through the C map
  const bool aux_al = args.aux != nullptr && (reinterpret_cast<uintptr_t>(args.aux) & 15) == 0;
  if (epi == EPI_RESID_F32 && aux_al && (reinterpret_cast<uintptr_t>(args.C) & 15) == 0 && (args.ldc % 4) == 0 &&
      (args.ldaux % 4) == 0 && make_map2(&tc, args.C, N, M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, true) &&
      make_map2(&td, args.aux, N, M, args.ldaux, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, true))
    args.c_tma = 1;
  if (epi == EPI_GELU && c_ok && args.D != nullptr && (reinterpret_cast<uintptr_t>(args.D) & 15) == 0 &&
      (args.ldd % 8) == 0 && make_map2(&tc, args.C, N, M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_map2(&td, args.D, N, M, args.ldd, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    args.c_tma = 1;
  if (epi == EPI_GELU_BWD && aux_al && c_ok && (args.ldaux % 8) == 0 &&
      make_map2(&tc, args.C, N, M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_map2(&td, args.aux, N, M, args.ldaux, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    args.c_tma = 1;
  if (epi == EPI_SWIGLU_BWD && aux_al && c_ok && (args.ldaux % 8) == 0 &&
      make_map2(&tc, args.C, 2 * (long long)N, M, args.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_map2(&td, args.aux, 2 * (long long)N, M, args.ldaux, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    args.c_tma = 1;
  const int tiles = num_m * num_n * splits;
  const int max_pairs = num_sms / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  return bn == 256 ? dispatch_pair<256>(epi, ta, tb, tc, td, args, 2 * pairs, stream)
                   : dispatch_pair<128>(epi, ta, tb, tc, td, args, 2 * pairs, stream);
}

// Grouped (mixture-of-experts) GEMM: validates the group description and runs the CTA-pair kernel
// with one split.  Mode 1 (rows): A is the expert-sorted activation buffer [M = capacity, K], K-major;
// B stacks grp_count expert blocks ([grp_count * N, K] K-major or [grp_count * K, N] MN-major, K a
// multiple of 64 so that no k-block reaches into the next expert); the bias, if any, stacks grp_count
// blocks of N.  Mode 2 (K, weight gradients): A [capacity, grp_m] and B [capacity, N] are both MN-major
// over the sorted buffer, C is [grp_count * grp_m, N] fp32 accumulated with EPI_RED_F32.
int pcb_gemm_grouped_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, int epi,
                            GemmArgs args, int num_sms, cudaStream_t stream) {
  if (args.grp_seg == nullptr || args.grp_count < 1 || args.grp_count > 4096) return -6;
  if ((reinterpret_cast<uintptr_t>(args.grp_seg) & 3) != 0) return -6;
  if (args.grp_mode == 1) {
    if (a_mn != 0 || args.M % 256 != 0) return -6;
    if (b_mn != 0 && args.K % 64 != 0) return -6;
    if (!(epi == EPI_F32 || epi == EPI_GELU || epi == EPI_GELU_BWD)) return -6;
    args.grp_b_off = b_mn ? args.K : args.N;
    args.grp_bias_off = args.N;
  } else if (args.grp_mode == 2) {
    if (a_mn != 1 || b_mn != 1 || args.grp_m <= 0 || args.grp_m % 256 != 0 ||
        (long long)args.M != (long long)args.grp_count * args.grp_m || args.K % 256 != 0)
      return -6;
    if (epi != EPI_RED_F32 || args.bias != nullptr) return -6;
  } else {
    return -6;
  }
  if (args.ag_world > 1 || args.rope_cs != nullptr) return -6;
  const int bn = args.N >= 256 ? 256 : 128;
  return pcb_gemm_pair_launch(A, a_mn, lda, B, b_mn, ldb, epi, args, bn, 1, num_sms, stream);
}
