// Causal flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference counterpart: PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs (attn_fwd: one
// block per (query, head), fp32 SIMT).  One CTA computes a 128-query tile of one (batch, head):
//
//   warp 4     TMA producer: Q once, then K_j / V_j 128-key tiles into a 2-stage ring
//   warp 5     MMA issuer:   S_j = Q K_j^T (M=128, N=128, K=hd) into one of two TMEM S buffers,
//                            then O_j = P_j V_j (M=128, N=hd, K=128) into one of two TMEM O buffers;
//                            S_{j+1} is issued before waiting for P_j, so QK^T overlaps the softmax
//   warps 0-3  softmax:      thread r owns query row r (TMEM lane r): row max over the S tile,
//                            p = exp((s - m) * scale) written as bf16 straight into the swizzled
//                            shared-memory layout the P operand descriptor expects, running sum l,
//                            and O accumulated in registers: O = O * exp((m_old - m) * scale) + O_j
//   epilogue   O / l in bf16, lse = m * scale + log(l) (the backward's convention)
//
// Heavy (late) query tiles are scheduled first.  Every wait is bounded and unwinds on timeout.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pcb {
namespace fa {

constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kThreads = 192;
constexpr int kAtom = 128 * 128;  // bytes of one [128 rows x 64 bf16] swizzled atom

template <int HD>
struct Cfg {
  static constexpr int ATOMS = HD / 64;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + ATOMS * kAtom;              // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * ATOMS * kAtom;          // 2 stages
  static constexpr int P_OFF = V_OFF + 2 * ATOMS * kAtom;          // 2 atoms (128 keys)
  static constexpr int BAR_OFF = P_OFF + 2 * kAtom;
  static constexpr int USED = BAR_OFF + 256;
  // keep one CTA per SM: a second CTA could not allocate its 512 TMEM columns anyway
  static constexpr int SMEM = (USED + 1024 > 120 * 1024 ? USED + 1024 : 120 * 1024);
};

PCB_DEVICE void fence_view_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, __nv_bfloat16* __restrict__ out, long long ld_o,
                       float* __restrict__ lse, int S, int H, float scale, int* err) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sP = smem + C::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* p_full = bars + 7;
  uint64_t* o_full = bars + 8;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;   // heavy tiles first
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int n_kv = qt + 1;                      // causal: key tiles 0..qt
  const int row0 = b * S + qt * kBQ;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(p_full, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) prefetch_tmap(&tm);
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(q_full, C::ATOMS * kAtom);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a) tma_load_2d(sQ + a * kAtom, &tm, q_full, h * HD + a * 64, row0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1u, err, kErrTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::ATOMS * kAtom);
        const int krow = b * S + j * kBKV;
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a) {
          tma_load_2d(sK + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (H + h) * HD + a * 64, krow);
          tma_load_2d(sV + (st * C::ATOMS + a) * kAtom, &tm, &kv_full[st], (2 * H + h) * HD + a * 64, krow);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16(kBQ, kBKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBQ, HD, 0, 1);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, err, kErrTimeoutFull, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, err, kErrTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + st * kBKV;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * kAtom + (k & 3) * 32;
          const uint64_t ad = make_smem_desc(q_addr + off, 16, 1024, 2);
          const uint64_t bd = make_smem_desc(k_addr + st * C::ATOMS * kAtom + off, 16, 1024, 2);
          umma_bf16(d, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        if (!mbar_wait(p_full, j & 1, err, kErrTimeoutTmemEmpty, abort_flag)) break;
        tc_fence_after();
        const int st = j & 1;
        const uint32_t d = tmem + 2 * kBKV + st * HD;
#pragma unroll
        for (int k = 0; k < kBKV / 16; ++k) {
          const uint64_t ad = make_smem_desc(p_addr + (k >> 2) * kAtom + (k & 3) * 32, 16, 1024, 2);
          const uint64_t bd = make_smem_desc(v_addr + st * C::ATOMS * kAtom + k * 2048, kAtom, 1024, 2);
          umma_bf16(d, ad, bd, idesc_o, k > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[st]);
        umma_commit(&kv_empty[st]);
      }
    }
  } else {
    // ---------------- softmax warps: one query row per thread ----------------
    const int r = threadIdx.x;                 // 0..127 == TMEM lane
    const int q = qt * kBQ + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m = -INFINITY, l = 0.f;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, err, kErrTimeoutTmemFull, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sbase = lane_base + st * kBKV;
      const bool diag = (j == qt);
      // pass 1: row max of this tile
      float tmax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kBKV / 32; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(sbase + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float s = __uint_as_float(u[e]);
          const bool valid = !diag || (c * 32 + e <= r);
          tmax = valid ? fmaxf(tmax, s) : tmax;
        }
      }
      const float m_new = fmaxf(m, tmax);
      const float corr = (m == -INFINITY) ? 0.f : __expf((m - m_new) * scale);
      const float msc = m_new * scale;
      // pass 2: probabilities -> bf16 P (swizzled K-major atoms), row sum
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < kBKV / 32; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(sbase + c * 32, u);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const bool v0 = !diag || (c * 32 + e <= r);
          const bool v1 = !diag || (c * 32 + e + 1 <= r);
          const float p0 = v0 ? __expf(__uint_as_float(u[e]) * scale - msc) : 0.f;
          const float p1 = v1 ? __expf(__uint_as_float(u[e + 1]) * scale - msc) : 0.f;
          rs += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        uint8_t* atom = sP + (c >> 1) * kAtom + r * 128;
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const int chunk = (c & 1) * 4 + e4;
          uint4 v = make_uint4(pk[4 * e4], pk[4 * e4 + 1], pk[4 * e4 + 2], pk[4 * e4 + 3]);
          *reinterpret_cast<uint4*>(atom + ((chunk ^ (r & 7)) << 4)) = v;
        }
      }
      l = l * corr + rs;
      m = m_new;
      fence_view_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // O_j = P_j V_j: fold into the register accumulator
      if (!mbar_wait(&o_full[st], (j >> 1) & 1, err, kErrTimeoutTmemFull, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t obase = lane_base + 2 * kBKV + st * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(obase + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c * 32 + e] = o[c * 32 + e] * corr + __uint_as_float(u[e]);
      }
    }
    if (ok) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (long long)(b * S + q) * ld_o + h * HD;
#pragma unroll
      for (int d = 0; d < HD; d += 8) {
        uint4 v = make_uint4(pack_bf16x2(o[d] * inv, o[d + 1] * inv), pack_bf16x2(o[d + 2] * inv, o[d + 3] * inv),
                             pack_bf16x2(o[d + 4] * inv, o[d + 5] * inv), pack_bf16x2(o[d + 6] * inv, o[d + 7] * inv));
        *reinterpret_cast<uint4*>(orow + d) = v;
      }
      lse[(long long)bh * S + q] = m * scale + logf(l);
    }
    tc_fence_before();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
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
  dim3 grid(S / fa::kBQ, B * H);
  fa::attn_fwd_tc_kernel<HD><<<grid, fa::kThreads, C::SMEM, s>>>(tm, reinterpret_cast<__nv_bfloat16*>(out), ld_o,
                                                                   lse, S, H, scale, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace pcb

// Same contract as pcb_attn_fwd (qkv [B*S, 3*H*HD] bf16 with q|k|v column blocks, out [B*S, H*HD]
// bf16, lse [B*H, S] fp32), on tcgen05.  S % 128 == 0, HD in {64, 128}, row strides % 8 == 0.
int pcb_attn_fwd_tc(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                    int HD, float scale, int* err, cudaStream_t s) {
  if (S % 128 != 0 || ld % 8 || ld_o % 8) return -1;
  if (reinterpret_cast<uintptr_t>(qkv) & 15) return -1;
  if (HD == 64) return pcb::fa_launch<64>(qkv, ld, out, ld_o, lse, B, S, H, scale, err, s);
  if (HD == 128) return pcb::fa_launch<128>(qkv, ld, out, ld_o, lse, B, S, H, scale, err, s);
  return -1;
}
