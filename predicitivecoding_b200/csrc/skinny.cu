// Skinny GEMM for decode-sized batches on the tcgen05 tensor cores: y[M, N] = x[M, K] @ W[K, N] with
// M <= 32 activation rows and a row-major [K, N] bf16 weight (the inference projection layout).
//
// A decode step is bound by reading the weights, so the kernel is laid out for HBM, not for the MMA:
// it computes the transposed product y^T = W^T x^T, so the weight's 128-column slice is the MMA's M (128
// TMEM lanes) and the activations are its N (32 columns), and it splits K over the S CTAs of a
// thread-block cluster (S = 1, 2, 4, 8 or 16) until about one CTA per SM streams a disjoint weight slab.
// Each CTA: one TMA producer thread loads [64 k x 128 n] weight tiles (MN-major, two 64-column boxes)
// and the matching [32 m x 64 k] activation tile into a 9-stage ring (the bytes in flight per SM bound a
// weight stream; a 4-stage ring with two CTAs per SM when that allows more CTAs), one thread issues tcgen05.mma (M 128, N 32, K 16 x 4) into 32 TMEM columns, and the
// four warps read the accumulator back (thread = weight column, registers = the 32 rows).  With S = 1 the
// rows are stored directly.  Otherwise CTA c of the cluster owns rows [c R, (c + 1) R), R = ceil(32 / S):
// every CTA pushes each owner its R rows with vector stores into the owner's shared memory (fire and
// forget), one cluster barrier makes them visible, and each owner sums its S partials in a fixed order
// and stores its rows -- no global workspace, no atomics, the same bits on every run, one barrier.
//
// A SwiGLU epilogue (W's columns in alternating blocks of 16 gate and 16 up columns, so each warp holds
// both halves of its 16 features) writes silu(gate) * up instead of the product; a RoPE epilogue takes a
// token's q | k | v, rotates q and k (partner column from the neighbouring lane) and appends k and v to
// the KV cache, so a decode step's qkv projection, RoPE and cache append are one launch.
//
// Launched as a programmatic dependent: the weights are not written by the kernels before it, so the
// first ring of weight tiles is requested (right after the barriers are initialised, while TMEM is being
// allocated) before griddepcontrol.wait and streams in while the previous kernel drains; activations
// and outputs are touched only after the wait.  Every mbarrier wait is bounded.
//
// Reference counterpart: PredictiveCoding.LLM/Infrastructure/GemmProvider.cs (the MatVec / MatMul used by
// GptModel.Step for each token) and PredictiveCoding.Device/Kernels/DeviceMath.cs (device GEMV).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace pcb {
namespace skinny {

constexpr int kBN = 128;                 // weight columns per CTA (MMA M)
constexpr int kBM = 32;                  // activation rows (MMA N)
constexpr int kBK = 64;
constexpr int kStagesWide = 9;           // 144 KB of weights in flight per CTA, one CTA per SM
constexpr int kStagesPair = 4;           // 64 KB per CTA, two CTAs per SM (twice the CTAs resident)
constexpr int kMaxSplits = 16;           // cluster size (above 8 where the GPU allows it)
constexpr int W_BYTES = kBK * kBN * 2;   // two [64 n x 64 k] boxes, 128B swizzle
constexpr int X_BYTES = kBM * kBK * 2;   // [32 m x 64 k], 128B swizzle
constexpr int STAGE = W_BYTES + X_BYTES;
// receive buffer of an owner: [S sources][128 columns][stride] fp32 holding its R = ceil(32 / S) rows;
// stride = R padded so that the accesses of consecutive columns hit disjoint banks (16-byte vectors of
// eight columns when R is a multiple of 4, single words of 32 columns otherwise)
__host__ __device__ constexpr int rows_per_owner(int S) { return (kBM + S - 1) / S; }
__host__ __device__ constexpr bool vec_rows(int S) { return rows_per_owner(S) % 4 == 0; }
__host__ __device__ constexpr int recv_stride(int S) {
  return vec_rows(S) ? (rows_per_owner(S) % 8 == 0 ? rows_per_owner(S) + 4 : rows_per_owner(S))
                     : (rows_per_owner(S) | 1);
}
__host__ __device__ constexpr int recv_bytes(int S) { return S == 1 ? 0 : S * kBN * recv_stride(S) * 4; }
__host__ __device__ constexpr int max_recv_bytes(int S = 2) {
  return S > kMaxSplits ? 0 : (recv_bytes(S) > max_recv_bytes(S + 1) ? recv_bytes(S) : max_recv_bytes(S + 1));
}
constexpr int RECV_MAX = max_recv_bytes();
template <int STAGES>
struct Layout {
  static constexpr int RECV_OFF = STAGES * STAGE;
  static constexpr int BAR_OFF = RECV_OFF + RECV_MAX;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
};
constexpr int kThreads = 128;
static_assert(Layout<kStagesWide>::SMEM <= 232448, "shared memory budget");
static_assert(2 * (Layout<kStagesPair>::SMEM + 1024) <= 233472, "two CTAs per SM");

struct Args {
  void* y;                 // [M, N] bf16 or fp32
  long long ldy;
  int M, N, K;
  int y_f32;
  int* err;
  unsigned long long* trace;  // optional: 8 globaltimer stamps (ns) per CTA at the phase boundaries
  int swiglu;                 // 1: W's columns alternate 16 gate / 16 up columns; y [M, N / 2] = silu(g) * u
  // RoPE + KV-cache append epilogue (rope_q != nullptr): the product is one token's q | k | v per row
  // (N = 3 H hd); q and k are rotated at position *pos (cs [cap, hd / 2] cos/sin pairs), q goes to
  // rope_q [M, H hd], k and v to row *pos of the caches [M, H, cap, hd]
  __nv_bfloat16* rope_q;
  __nv_bfloat16* rope_k;
  __nv_bfloat16* rope_v;
  const float2* rope_cs;
  const long long* pos;
  int heads, hd, cap;
};

PCB_DEVICE unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

PCB_DEVICE void st_dsmem_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
PCB_DEVICE void st_dsmem_b32(uint32_t addr, uint32_t a) {
  asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(addr), "r"(a) : "memory");
}

PCB_DEVICE void store_out(const Args& a, int m, int n, float v) {
  if (a.y_f32) reinterpret_cast<float*>(a.y)[(long long)m * a.ldy + n] = v;
  else reinterpret_cast<__nv_bfloat16*>(a.y)[(long long)m * a.ldy + n] = __float2bfloat16_rn(v);
}

// Store of row m's value v in column n (thread = column, a warp = 32 aligned columns).  With the SwiGLU
// epilogue a warp's columns are 16 gate columns then the 16 matching up columns: lanes 0-15 take the up
// value from lane + 16 and store silu(gate) * up as feature (n / 32) * 16 + lane.  Every lane of the warp
// must call it (the shuffle); `ok` guards the store.
PCB_DEVICE void store_act(const Args& a, int m, int n, float v, bool ok) {
  if (a.rope_q != nullptr) {
    // adjacent columns (lanes 2j, 2j + 1) are the pair (x_2j, x_2j+1) that RoPE rotates together
    const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
    if (!ok) return;
    const int D = a.heads * a.hd, part = n / D, within = n - part * D;
    const int h = within / a.hd, d = within - h * a.hd;
    const long long p = *a.pos;
    if (part == 2) {
      a.rope_v[(((long long)m * a.heads + h) * a.cap + p) * a.hd + d] = __float2bfloat16_rn(v);
      return;
    }
    const float2 c = a.rope_cs[p * (a.hd / 2) + d / 2];
    const float r = (d & 1) ? partner * c.y + v * c.x : v * c.x - partner * c.y;
    if (part == 0) a.rope_q[(long long)m * D + within] = __float2bfloat16_rn(r);
    else a.rope_k[(((long long)m * a.heads + h) * a.cap + p) * a.hd + d] = __float2bfloat16_rn(r);
    return;
  }
  if (!a.swiglu) {
    if (ok) store_out(a, m, n, v);
    return;
  }
  const float up = __shfl_down_sync(0xffffffffu, v, 16);
  const int lane = threadIdx.x & 31;
  if (ok && lane < 16) store_out(a, m, (n >> 5) * 16 + lane, v / (1.f + __expf(-v)) * up);
}

template <int S, int kStages>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const Args a) {
  constexpr int R = rows_per_owner(S);       // rows each CTA of the cluster stores (the last ones may have fewer)
  constexpr int STRIDE = recv_stride(S);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using L = Layout<kStages>;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* recv = reinterpret_cast<float*>(smem + L::RECV_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile = blockIdx.x, split = blockIdx.y;   // the cluster spans blockIdx.y: rank == split
  const int n0 = ntile * kBN;
  const int total_kb = (a.K + kBK - 1) / kBK;
  const int kb0 = split * total_kb / S;
  const int kb1 = (split + 1) * total_kb / S;
  const int nkb = kb1 - kb0;
  const int pre = min(nkb, kStages);
  unsigned long long* tr = a.trace ? a.trace + 8ull * (blockIdx.y * gridDim.x + blockIdx.x) : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = global_ns();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
    // the first ring of weight tiles does not depend on the previous kernel: request it now
    for (int i = 0; i < pre; ++i) {
      uint8_t* sw = smem + i * STAGE;
      mbar_arrive_expect_tx(&full[i], STAGE);
      tma_load_2d(sw, &tmW, &full[i], n0, (kb0 + i) * kBK);
      tma_load_2d(sw + 8192, &tmW, &full[i], n0 + 64, (kb0 + i) * kBK);
    }
    if (tr) tr[1] = global_ns();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tr && threadIdx.x == 0) tr[2] = global_ns();
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    for (int i = 0; i < pre; ++i) tma_load_2d(smem + i * STAGE + W_BYTES, &tmX, &full[i], (kb0 + i) * kBK, 0);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % kStages, kb = kb0 + i;
      if (!mbar_wait(&empty[s], ((i / kStages) & 1) ^ 1u, a.err, kErrTimeoutEmpty, abort_flag)) break;
      uint8_t* sw = smem + s * STAGE;
      mbar_arrive_expect_tx(&full[s], STAGE);
      tma_load_2d(sw, &tmW, &full[s], n0, kb * kBK);
      tma_load_2d(sw + 8192, &tmW, &full[s], n0 + 64, kb * kBK);
      tma_load_2d(sw + W_BYTES, &tmX, &full[s], kb * kBK, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = make_idesc_bf16(kBN, kBM, 1, 0);   // A = W^T (MN-major), B = x (K-major)
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&full[s], (i / kStages) & 1, a.err, kErrTimeoutFull, abort_flag)) break;
      if (tr && i == 0) tr[3] = global_ns();
      tc_fence_after();
      const uint32_t sw = smem_u32(smem + s * STAGE);
      const uint32_t sx = sw + W_BYTES;
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        umma_bf16(tmem, make_smem_desc(sw + k * 2048, 8192, 1024, 2), make_smem_desc(sx + k * 32, 16, 1024, 2),
                  idesc, (i > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();

  // ---------------- epilogue: thread = weight column n0 + threadIdx.x, registers = the 32 rows ----------------
  // lanes spin independently: agree on the outcome (and reconverge) before the warp-collective tcgen05.ld
  const bool got = __all_sync(0xffffffffu, mbar_wait(done, 0, a.err, kErrTimeoutTmemFull, abort_flag) &&
                                               !*abort_flag && nkb > 0);
  tc_fence_after();
  uint32_t r[32];
  tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16), r);
  tmem_ld_wait();
  if (!got) {
#pragma unroll
    for (int m = 0; m < kBM; ++m) r[m] = 0u;   // no k-blocks (or an abort): this split adds nothing
  }
  if (tr && threadIdx.x == 0) tr[4] = global_ns();
  const int n = n0 + threadIdx.x;
  if constexpr (S == 1) {
#pragma unroll
    for (int m = 0; m < kBM; ++m)
      if (m < a.M) store_act(a, m, n, __uint_as_float(r[m]), n < a.N);   // m < M is warp-uniform
  } else {
    // push rows [c R, (c + 1) R) to owner c, at [split][column][row - c R] of its receive buffer
    const uint32_t mine = smem_u32(recv) + (uint32_t)((split * kBN + threadIdx.x) * STRIDE * 4);
#pragma unroll
    for (int c = 0; c < S; ++c) {
      if (c * R < kBM && c * R < a.M) {
        const uint32_t dst = mapa_shared(mine, (uint32_t)c);
        if constexpr (vec_rows(S)) {
#pragma unroll
          for (int j = 0; j < R; j += 4)
            if (c * R + j < kBM)
              st_dsmem_v4(dst + j * 4, r[c * R + j], r[c * R + j + 1], r[c * R + j + 2], r[c * R + j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < R; ++j)
            if (c * R + j < kBM) st_dsmem_b32(dst + j * 4, r[c * R + j]);
        }
      }
    }
    cluster_sync_all();   // release the pushes / acquire the partials addressed to this CTA
    if (tr && threadIdx.x == 0) tr[5] = global_ns();
    if (split * R < a.M) {                                      // uniform over the CTA
      float acc[R];
#pragma unroll
      for (int j = 0; j < R; ++j) acc[j] = 0.f;
#pragma unroll
      for (int q = 0; q < S; ++q) {                            // source CTAs in order: deterministic
        const float* src = recv + (q * kBN + threadIdx.x) * STRIDE;
        if constexpr (vec_rows(S)) {
#pragma unroll
          for (int j = 0; j < R; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(src + j);
            acc[j] += v.x;
            acc[j + 1] += v.y;
            acc[j + 2] += v.z;
            acc[j + 3] += v.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < R; ++j) acc[j] += src[j];
        }
      }
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (split * R + j < a.M && split * R + j < kBM) store_act(a, split * R + j, n, acc[j], n < a.N);
    }
    if (tr && threadIdx.x == 0) tr[6] = global_ns();
  }
  if (tr && threadIdx.x == 0) tr[7] = global_ns();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 32);
}

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

static bool make_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t bi,
                     uint32_t bo) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {bi, bo};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace skinny
}  // namespace pcb

using namespace pcb;

#include "skinny_api.h"

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const skinny::Args);

// kernel for cluster size S (1, 2, 4, 8, 16) and ring depth (pair: 4 stages, two CTAs per SM)
static KernelFn skinny_fn(int S, bool pair) {
  switch (S) {
    case 1: return pair ? skinny::skinny_kernel<1, skinny::kStagesPair> : skinny::skinny_kernel<1, skinny::kStagesWide>;
    case 2: return pair ? skinny::skinny_kernel<2, skinny::kStagesPair> : skinny::skinny_kernel<2, skinny::kStagesWide>;
    case 4: return pair ? skinny::skinny_kernel<4, skinny::kStagesPair> : skinny::skinny_kernel<4, skinny::kStagesWide>;
    case 8: return pair ? skinny::skinny_kernel<8, skinny::kStagesPair> : skinny::skinny_kernel<8, skinny::kStagesWide>;
    default:
      return pair ? skinny::skinny_kernel<16, skinny::kStagesPair> : skinny::skinny_kernel<16, skinny::kStagesWide>;
  }
}
static int skinny_smem(bool pair) {
  return pair ? skinny::Layout<skinny::kStagesPair>::SMEM : skinny::Layout<skinny::kStagesWide>::SMEM;
}

static void skinny_attrs() {
  static std::once_flag once;
  std::call_once(once, [] {
    for (int S = 1; S <= skinny::kMaxSplits; S *= 2)
      for (int pair = 0; pair < 2; ++pair) {
        cudaFuncSetAttribute(skinny_fn(S, pair), cudaFuncAttributeMaxDynamicSharedMemorySize, skinny_smem(pair));
        cudaFuncSetAttribute(skinny_fn(S, pair), cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      }
    cudaGetLastError();
  });
}

// Clusters of `S` CTAs the GPU can hold at once for a ring depth; cached per device.
static int skinny_max_clusters(int S, bool pair) {
  static int cache[64][2][skinny::kMaxSplits + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  int& c = cache[dev][pair ? 1 : 0][S];
  if (c == 0) {
    skinny_attrs();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, S, 1);
    cfg.blockDim = dim3(skinny::kThreads, 1, 1);
    cfg.dynamicSmemBytes = skinny_smem(pair);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = S;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, skinny_fn(S, pair), &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    c = n > 0 ? n : -1;
  }
  return c;
}

// Split count (cluster size) and ring depth for a skinny product: a power of two up to 16 so that column
// tiles x splits fill about one wave (one CTA per SM with the deep ring, two with the shallow one), each
// split has at least two k-blocks, and all the clusters (one per column tile) are resident together; the
// shallow ring is taken when it allows a larger cluster.  (Clusters of 3, 6 or 9 CTAs, which fill more
// SMs for some shapes, measured slower on B200: 9.2 against 4.0 us for a [32 x 768] x [768 x 2304]
// product with 6 against 4, 10.1 against 5.3 us for [32 x 2048] x [2048 x 2048] with 9 against 4.)
// Returns splits, negated when the shallow ring is chosen.
static int skinny_pick(int N, int K, int num_sms, bool pair) {
  const int ntiles = (N + skinny::kBN - 1) / skinny::kBN;
  const int total_kb = (K + skinny::kBK - 1) / skinny::kBK;
  const int slots = pair ? 2 * num_sms : num_sms;
  const int cap = min(min(max(1, slots / ntiles), max(1, total_kb / 2)), skinny::kMaxSplits);
  int s = 1;
  while (s * 2 <= cap) s *= 2;
  while (s > 1 && skinny_max_clusters(s, pair) < ntiles) s /= 2;
  return s;
}

int pcb_skinny_splits(int N, int K, int num_sms) {
  const char* e = getenv("PCB_SKINNY_RING");           // "wide" / "pair" force one ring depth
  const bool only_wide = e && e[0] == 'w', only_pair = e && e[0] == 'p';
  const int wide = skinny_pick(N, K, num_sms, false);
  if (only_wide) return wide;
  const int pair = skinny_pick(N, K, num_sms, true);
  // more column tiles than SMs (an LM head): the shallow ring keeps them in one wave
  // (32 x 2048 x 32000: 23.0 us against 31.3 us on the deep ring and 29.0 us on the regular GEMM)
  const bool many_tiles = (N + skinny::kBN - 1) / skinny::kBN > num_sms;
  return (only_pair || many_tiles || pair > wide) ? -pair : wide;
}

// Programmatic dependent launch (PCB_PDL=0 turns it off).
static bool skinny_pdl() {
  static const bool on = [] {
    const char* e = getenv("PCB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// y [M, N] (bf16, or fp32 with y_f32) = x [M, K] bf16 @ W [K, N] bf16 (row-major), M <= 32, K split over
// `splits` CTAs of a cluster (1, 2, 4, 8 or 16; negative: the same count on the shallow two-CTAs-per-SM
// ring); `trace` (optional) receives 8 timestamps per CTA; `swiglu`: W's columns alternate 16 gate and 16
// up columns (N a multiple of 32) and y [M, N / 2] receives silu(gate) * up; `rope` (optional): the
// product is q | k | v of one token per row, rotated and written to rope->q and the caches (y unused).
// Returns 0, -1 bad arguments, -5 tensor-map encode, -(1000 + cudaError) launch.
int pcb_skinny_gemm(const void* x, long long ldx, const void* w, long long ldw, void* y, long long ldy, int y_f32,
                    int M, int N, int K, int splits, int* err, unsigned long long* trace, int swiglu,
                    const SkinnyRope* rope, cudaStream_t stream) {
  if (M < 1 || M > skinny::kBM || N < 1 || K < 1) return -1;
  const bool pair = splits < 0;
  if (pair) splits = -splits;
  if (splits != 1 && splits != 2 && splits != 4 && splits != 8 && splits != 16) return -1;
  if (ldx % 8 || ldw % 8 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)) return -1;
  CUtensorMap tw, tx;
  if (!skinny::make_map(&tw, w, (uint64_t)N, (uint64_t)K, (uint64_t)ldw, 64, 64)) return -5;
  if (!skinny::make_map(&tx, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, 64, skinny::kBM)) return -5;
  skinny::Args a{};
  a.y = y;
  a.ldy = ldy;
  a.M = M;
  a.N = N;
  a.K = K;
  a.y_f32 = y_f32;
  a.err = err;
  a.trace = trace;
  if (swiglu && N % 32) return -1;
  a.swiglu = swiglu ? 1 : 0;
  if (rope != nullptr) {
    if (swiglu || N != 3 * rope->heads * rope->hd || rope->hd % 2) return -1;
    a.rope_q = rope->q;
    a.rope_k = rope->k;
    a.rope_v = rope->v;
    a.rope_cs = reinterpret_cast<const float2*>(rope->cs);
    a.pos = rope->pos;
    a.heads = rope->heads;
    a.hd = rope->hd;
    a.cap = rope->cap;
  }
  skinny_attrs();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + skinny::kBN - 1) / skinny::kBN, splits, 1);
  cfg.blockDim = dim3(skinny::kThreads, 1, 1);
  cfg.dynamicSmemBytes = skinny_smem(pair);
  cfg.stream = stream;
  cudaLaunchAttribute attr_v[2];
  attr_v[0].id = cudaLaunchAttributeClusterDimension;
  attr_v[0].val.clusterDim.x = 1;
  attr_v[0].val.clusterDim.y = splits;
  attr_v[0].val.clusterDim.z = 1;
  attr_v[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_v[1].val.programmaticStreamSerializationAllowed = skinny_pdl() ? 1 : 0;
  cfg.attrs = attr_v;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_fn(splits, pair), tw, tx, a);
  return e == cudaSuccess ? 0 : -(1000 + (int)e);
}
