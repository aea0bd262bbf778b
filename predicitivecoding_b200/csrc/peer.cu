// Peer-memory collectives over NVLink / NVSwitch, fused with the optimizer.
//
// The reference's "NCCL" is a host mock over float[][] (PredictiveCoding.Device/Nccl/NcclProvider.cs:1-109)
// and its data parallelism is CPU replicas (PredictiveCoding.LLM/Training/Trainer.cs:118-194).  Here each
// rank exposes its gradient and bf16-weight buffers to every peer through CUDA IPC; kernels read and write
// peer memory directly with SM loads/stores over NVLink:
//
//   rs_adamw_ag:  for the owned shard of a parameter range, sum the gradient over all ranks (reduce-
//                 scatter), apply AdamW to the local fp32 master / moments, and store the new bf16 weights
//                 into every rank's working copy (all-gather) -- one pass, no intermediate buffers.
//   pc_allreduce_update: sum a delta over all ranks for the owned shard and apply W += a*sum, decay,
//                 then push fp32 and bf16 weights to every peer (the PC-MLP Hebbian update).
//   peer_barrier: bounded flag barrier (release/acquire at system scope) that orders the collective
//                 against the producers and consumers on every rank.
//
// No TMA and no multicast loads are used on peer memory: only plain ld/st.  Every wait is bounded;
// on timeout the kernel records an error code in a device word and returns.
#include <cstdint>
#include <cstdio>

#include "common.cuh"

namespace pcb {

PCB_DEVICE void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
PCB_DEVICE unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags: every rank owns an array flags[world] in its own memory; peers write their slot.
// ctr: local epoch counter (device memory) so the same launch works under CUDA-graph replay.
__global__ void peer_barrier_kernel(unsigned int* const* __restrict__ peer_flags, unsigned int* __restrict__ ctr,
                                    int rank, int world, int* __restrict__ err) {
  __shared__ unsigned int epoch;
  if (threadIdx.x == 0) {
    __threadfence_system();
    epoch = *ctr + 1;
    *ctr = epoch;
  }
  __syncthreads();
  const unsigned int e = epoch;
  const int p = threadIdx.x;
  if (p < world) st_release_sys(peer_flags[p] + rank, e);
  if (p < world) {
    const unsigned int* mine = peer_flags[rank] + p;
    const long long t0 = clock64();
    while (ld_acquire_sys(mine) < e) {
      if (clock64() - t0 > kSpinBudgetCycles) {
        record_error(err, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
}

// Sum over ranks of grad[i] for i in [lo, hi) (global arena indices), AdamW on the local shard
// state (index i - lo), and push bf16(w) into every rank's working copy at index i.
// hyper = [lr, wd, bc1, bc2, grad_scale]; weight decay applies to i < n_decay.
template <int WORLD>
__global__ void __launch_bounds__(256)
    rs_adamw_ag_kernel(const float* const* __restrict__ grad_peers, __nv_bfloat16* const* __restrict__ w16_peers,
                       float* __restrict__ w32, float* __restrict__ m, float* __restrict__ v, long long lo,
                       long long hi, long long n_decay, const float* __restrict__ hyper, float b1, float b2,
                       float eps, int world_rt) {
  const int world = WORLD > 0 ? WORLD : world_rt;
  const float lr = hyper[0], wd = hyper[1], bc1 = hyper[2], bc2 = hyper[3], gs = hyper[4];
  const long long n4 = (hi - lo) / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n4; q += (long long)gridDim.x * blockDim.x) {
    const long long i = lo + 4 * q;
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int p = 0; p < world; ++p) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(grad_peers[p] + i));
      g.x += x.x; g.y += x.y; g.z += x.z; g.w += x.w;
    }
    const long long j = 4 * q;
    float4 w = *reinterpret_cast<float4*>(w32 + j);
    float4 mm = *reinterpret_cast<float4*>(m + j);
    float4 vv = *reinterpret_cast<float4*>(v + j);
    float gg[4] = {g.x, g.y, g.z, g.w}, ww[4] = {w.x, w.y, w.z, w.w};
    float m4[4] = {mm.x, mm.y, mm.z, mm.w}, v4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float gi = isfinite(gg[k]) ? gg[k] * gs : 0.f;
      m4[k] = b1 * m4[k] + (1.f - b1) * gi;
      v4[k] = b2 * v4[k] + (1.f - b2) * gi * gi;
      ww[k] -= lr * (m4[k] / bc1) / (sqrtf(v4[k] / bc2) + eps);
      if (i + k < n_decay) ww[k] -= lr * wd * ww[k];
    }
    *reinterpret_cast<float4*>(w32 + j) = make_float4(ww[0], ww[1], ww[2], ww[3]);
    *reinterpret_cast<float4*>(m + j) = make_float4(m4[0], m4[1], m4[2], m4[3]);
    *reinterpret_cast<float4*>(v + j) = make_float4(v4[0], v4[1], v4[2], v4[3]);
    uint2 packed;
    packed.x = pack_bf16x2(ww[0], ww[1]);
    packed.y = pack_bf16x2(ww[2], ww[3]);
#pragma unroll 8
    for (int p = 0; p < world; ++p) *reinterpret_cast<uint2*>(w16_peers[p] + i) = packed;
  }
}

// PC data-parallel weight update: for i in [lo, hi): W[i] = (W[i] + alpha * sum_p delta_p[i]) * decay,
// written to every rank's fp32 W and bf16 copy (all ranks hold full weights).
__global__ void __launch_bounds__(256)
    pc_allreduce_update_kernel(const float* const* __restrict__ delta_peers, float* const* __restrict__ w_peers,
                               __nv_bfloat16* const* __restrict__ w16_peers, long long lo, long long hi, float alpha,
                               float decay, int world, int rank) {
  const long long n4 = (hi - lo) / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n4; q += (long long)gridDim.x * blockDim.x) {
    const long long i = lo + 4 * q;
    float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(delta_peers[p] + i));
      d.x += x.x; d.y += x.y; d.z += x.z; d.w += x.w;
    }
    // every rank's W is identical; read the local copy
    float4 w = __ldcg(reinterpret_cast<const float4*>(w_peers[rank] + i));
    w.x = (w.x + alpha * d.x) * decay;
    w.y = (w.y + alpha * d.y) * decay;
    w.z = (w.z + alpha * d.z) * decay;
    w.w = (w.w + alpha * d.w) * decay;
    uint2 packed;
    packed.x = pack_bf16x2(w.x, w.y);
    packed.y = pack_bf16x2(w.z, w.w);
    for (int p = 0; p < world; ++p) {
      *reinterpret_cast<float4*>(w_peers[p] + i) = w;
      if (w16_peers != nullptr) *reinterpret_cast<uint2*>(w16_peers[p] + i) = packed;
    }
  }
}

// Sum of `world` peer buffers into a local output for [lo, hi) (reduce-scatter without the optimizer;
// used by tests and by the generic all-reduce).  If `out_peers` is given the sum is pushed to every rank.
__global__ void __launch_bounds__(256)
    peer_reduce_kernel(const float* const* __restrict__ in_peers, float* const* __restrict__ out_peers,
                       long long lo, long long hi, float scale, int world) {
  const long long n4 = (hi - lo) / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n4; q += (long long)gridDim.x * blockDim.x) {
    const long long i = lo + 4 * q;
    float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(in_peers[p] + i));
      d.x += x.x; d.y += x.y; d.z += x.z; d.w += x.w;
    }
    d.x *= scale; d.y *= scale; d.z *= scale; d.w *= scale;
    for (int p = 0; p < world; ++p) *reinterpret_cast<float4*>(out_peers[p] + i) = d;
  }
}

// ---------------------------------------------------------------------------------------------
// Bucketed data-parallel optimizer step (gradient reduce-scatter overlapped with the backward).
//
// Every rank owns piece `rank` of every gradient bucket.  During the backward each rank's copy
// engines push its gradient pieces into the owners' staging buffers (slot = source rank, in the
// owner's local order), so the transfer costs no SM time and overlaps the remaining backward.
// After one barrier the owner runs
//   dp_reduce_sumsq: g = own gradient + sum of the staged slots, non-finite -> 0, kept in gshard,
//                    and the sum of squares accumulated in double (for global-norm clipping);
//   dp_norm_push:    its partial sum of squares stored into every rank's slot table;
//   dp_adamw_ag:     clip scale from the summed table, AdamW on the local master shard (decay only
//                    below each bucket's decay end), bf16 weights stored into every rank's copy.
// The table `tab` holds one row per bucket: (local offset, flat start of my piece, length, flat
// decay end); lengths and offsets are multiples of 64 elements.
constexpr int kDpMaxBuckets = 128;

PCB_DEVICE int dp_find(const long long* tab, int nb, long long j) {
  int lo = 0, hi = nb - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab[4 * mid] <= j) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int WORLD>
__global__ void __launch_bounds__(256)
    dp_reduce_sumsq_kernel(const float* __restrict__ grad, const float* __restrict__ staging, long long shard,
                           const long long* __restrict__ tab_g, int nb, int rank, int world_rt,
                           float* __restrict__ gshard, double* __restrict__ sumsq) {
  const int world = WORLD > 0 ? WORLD : world_rt;
  __shared__ long long tab[4 * kDpMaxBuckets];
  __shared__ float part[8];
  for (int t = threadIdx.x; t < 4 * nb; t += blockDim.x) tab[t] = tab_g[t];
  __syncthreads();
  float acc = 0.f;
  const long long n4 = shard / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n4; q += (long long)gridDim.x * blockDim.x) {
    const long long j = 4 * q;
    const int b = dp_find(tab, nb, j);
    const long long i = tab[4 * b + 1] + (j - tab[4 * b]);
    float4 g = __ldcs(reinterpret_cast<const float4*>(grad + i));
#pragma unroll 8
    for (int p = 0; p < world; ++p) {
      if (p == rank) continue;
      const float4 x = __ldcs(reinterpret_cast<const float4*>(staging + (long long)p * shard + j));
      g.x += x.x; g.y += x.y; g.z += x.z; g.w += x.w;
    }
    g.x = isfinite(g.x) ? g.x : 0.f;
    g.y = isfinite(g.y) ? g.y : 0.f;
    g.z = isfinite(g.z) ? g.z : 0.f;
    g.w = isfinite(g.w) ? g.w : 0.f;
    *reinterpret_cast<float4*>(gshard + j) = g;
    acc += g.x * g.x + g.y * g.y + g.z * g.z + g.w * g.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    atomicAdd(sumsq, (double)t);
  }
}

__global__ void dp_norm_push_kernel(const double* __restrict__ sumsq, double* const* __restrict__ slot_peers, int rank,
                                    int world) {
  const int p = threadIdx.x;
  if (p < world) {
    *reinterpret_cast<volatile double*>(slot_peers[p] + rank) = *sumsq;
    __threadfence_system();
  }
}

template <int WORLD>
__global__ void __launch_bounds__(256)
    dp_adamw_ag_kernel(const float* __restrict__ gshard, float* __restrict__ w32, float* __restrict__ m,
                       float* __restrict__ v, __nv_bfloat16* const* __restrict__ w16_peers, long long shard,
                       const long long* __restrict__ tab_g, int nb, const float* __restrict__ hyper, float b1,
                       float b2, float eps, const double* __restrict__ norm_slots, float max_norm, int world_rt) {
  const int world = WORLD > 0 ? WORLD : world_rt;
  __shared__ long long tab[4 * kDpMaxBuckets];
  for (int t = threadIdx.x; t < 4 * nb; t += blockDim.x) tab[t] = tab_g[t];
  __syncthreads();
  const float lr = hyper[0], wd = hyper[1], bc1 = hyper[2], bc2 = hyper[3];
  float s = hyper[4];
  if (norm_slots != nullptr && max_norm > 0.f) {   // global norm of the mean gradient, as the reference clips
    double t = 0.0;
    for (int p = 0; p < world; ++p) t += norm_slots[p];
    const float norm = static_cast<float>(sqrt(t)) * s;
    if (norm > max_norm) s *= max_norm / (norm + 1e-6f);
  }
  const long long n4 = shard / 4;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n4; q += (long long)gridDim.x * blockDim.x) {
    const long long j = 4 * q;
    const int b = dp_find(tab, nb, j);
    const long long i = tab[4 * b + 1] + (j - tab[4 * b]);
    const long long dend = tab[4 * b + 3];
    const float4 g = __ldcs(reinterpret_cast<const float4*>(gshard + j));
    float4 w = *reinterpret_cast<float4*>(w32 + j);
    float4 mm = *reinterpret_cast<float4*>(m + j);
    float4 vv = *reinterpret_cast<float4*>(v + j);
    float gg[4] = {g.x, g.y, g.z, g.w}, ww[4] = {w.x, w.y, w.z, w.w};
    float m4[4] = {mm.x, mm.y, mm.z, mm.w}, v4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gi = gg[k] * s;
      m4[k] = b1 * m4[k] + (1.f - b1) * gi;
      v4[k] = b2 * v4[k] + (1.f - b2) * gi * gi;
      ww[k] -= lr * (m4[k] / bc1) / (sqrtf(v4[k] / bc2) + eps);
      if (i + k < dend) ww[k] -= lr * wd * ww[k];
    }
    *reinterpret_cast<float4*>(w32 + j) = make_float4(ww[0], ww[1], ww[2], ww[3]);
    *reinterpret_cast<float4*>(m + j) = make_float4(m4[0], m4[1], m4[2], m4[3]);
    *reinterpret_cast<float4*>(v + j) = make_float4(v4[0], v4[1], v4[2], v4[3]);
    uint2 packed;
    packed.x = pack_bf16x2(ww[0], ww[1]);
    packed.y = pack_bf16x2(ww[2], ww[3]);
#pragma unroll 8
    for (int p = 0; p < world; ++p) *reinterpret_cast<uint2*>(w16_peers[p] + i) = packed;
  }
}

}  // namespace pcb

using namespace pcb;

// ------------------------------------------------------------------ host API
int pcb_peer_alloc(size_t bytes, void** ptr) {
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return -3;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return -3;
  return 0;
}
int pcb_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : -3; }
int pcb_ipc_handle(void* ptr, void* out64) {
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -3;
  memcpy(out64, &h, sizeof(h));
  return 0;
}
int pcb_ipc_open(const void* in64, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, in64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : -3;
}
int pcb_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : -3; }

int pcb_peer_barrier(void* const* peer_flags_dev, unsigned int* ctr, int rank, int world, int* err, cudaStream_t s) {
  if (world > 32) return -1;
  peer_barrier_kernel<<<1, 32, 0, s>>>(reinterpret_cast<unsigned int* const*>(peer_flags_dev), ctr, rank, world, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

static int grid_for_n4(long long n4, int num_sms) {
  long long b = (n4 + 255) / 256;
  const long long cap = (long long)(num_sms > 0 ? num_sms : 148) * 4;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

int pcb_rs_adamw_ag(void* const* grad_peers, void* const* w16_peers, float* w32, float* m, float* v, long long lo,
                    long long hi, long long n_decay, const float* hyper, float b1, float b2, float eps, int world,
                    int num_sms, cudaStream_t s) {
  if ((lo % 4) || ((hi - lo) % 4)) return -1;
  const int grid = grid_for_n4((hi - lo) / 4, num_sms);
  auto gp = reinterpret_cast<const float* const*>(grad_peers);
  auto wp = reinterpret_cast<__nv_bfloat16* const*>(w16_peers);
  switch (world) {
    case 2: rs_adamw_ag_kernel<2><<<grid, 256, 0, s>>>(gp, wp, w32, m, v, lo, hi, n_decay, hyper, b1, b2, eps, world); break;
    case 4: rs_adamw_ag_kernel<4><<<grid, 256, 0, s>>>(gp, wp, w32, m, v, lo, hi, n_decay, hyper, b1, b2, eps, world); break;
    case 8: rs_adamw_ag_kernel<8><<<grid, 256, 0, s>>>(gp, wp, w32, m, v, lo, hi, n_decay, hyper, b1, b2, eps, world); break;
    default: rs_adamw_ag_kernel<0><<<grid, 256, 0, s>>>(gp, wp, w32, m, v, lo, hi, n_decay, hyper, b1, b2, eps, world);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_pc_allreduce_update(void* const* delta_peers, void* const* w_peers, void* const* w16_peers, long long lo,
                            long long hi, float alpha, float decay, int world, int rank, int num_sms, cudaStream_t s) {
  if ((lo % 4) || ((hi - lo) % 4)) return -1;
  const int grid = grid_for_n4((hi - lo) / 4, num_sms);
  pc_allreduce_update_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float* const*>(delta_peers),
                                                  reinterpret_cast<float* const*>(w_peers),
                                                  reinterpret_cast<__nv_bfloat16* const*>(w16_peers), lo, hi, alpha,
                                                  decay, world, rank);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_peer_reduce(void* const* in_peers, void* const* out_peers, long long lo, long long hi, float scale, int world,
                    int num_sms, cudaStream_t s) {
  if ((lo % 4) || ((hi - lo) % 4)) return -1;
  const int grid = grid_for_n4((hi - lo) / 4, num_sms);
  peer_reduce_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float* const*>(in_peers),
                                          reinterpret_cast<float* const*>(out_peers), lo, hi, scale, world);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// ------------------------------------------------------------------ bucketed data-parallel step
int pcb_dp_reduce_sumsq(const float* grad, const float* staging, long long shard, const long long* tab, int nb,
                        int rank, int world, float* gshard, double* sumsq, int num_sms, cudaStream_t s) {
  if (nb <= 0 || nb > kDpMaxBuckets || (shard % 4)) return -1;
  const int grid = grid_for_n4(shard / 4, num_sms);
  switch (world) {
    case 2: dp_reduce_sumsq_kernel<2><<<grid, 256, 0, s>>>(grad, staging, shard, tab, nb, rank, world, gshard, sumsq); break;
    case 4: dp_reduce_sumsq_kernel<4><<<grid, 256, 0, s>>>(grad, staging, shard, tab, nb, rank, world, gshard, sumsq); break;
    case 8: dp_reduce_sumsq_kernel<8><<<grid, 256, 0, s>>>(grad, staging, shard, tab, nb, rank, world, gshard, sumsq); break;
    default: dp_reduce_sumsq_kernel<0><<<grid, 256, 0, s>>>(grad, staging, shard, tab, nb, rank, world, gshard, sumsq);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_dp_norm_push(const double* sumsq, void* const* slot_peers, int rank, int world, cudaStream_t s) {
  if (world > 1024) return -1;
  dp_norm_push_kernel<<<1, 32 * ((world + 31) / 32), 0, s>>>(sumsq, reinterpret_cast<double* const*>(slot_peers),
                                                             rank, world);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_dp_adamw_ag(const float* gshard, float* w32, float* m, float* v, void* const* w16_peers, long long shard,
                    const long long* tab, int nb, const float* hyper, float b1, float b2, float eps,
                    const double* norm_slots, float max_norm, int world, int num_sms, cudaStream_t s) {
  if (nb <= 0 || nb > kDpMaxBuckets || (shard % 4)) return -1;
  const int grid = grid_for_n4(shard / 4, num_sms);
  auto wp = reinterpret_cast<__nv_bfloat16* const*>(w16_peers);
  switch (world) {
    case 2: dp_adamw_ag_kernel<2><<<grid, 256, 0, s>>>(gshard, w32, m, v, wp, shard, tab, nb, hyper, b1, b2, eps, norm_slots, max_norm, world); break;
    case 4: dp_adamw_ag_kernel<4><<<grid, 256, 0, s>>>(gshard, w32, m, v, wp, shard, tab, nb, hyper, b1, b2, eps, norm_slots, max_norm, world); break;
    case 8: dp_adamw_ag_kernel<8><<<grid, 256, 0, s>>>(gshard, w32, m, v, wp, shard, tab, nb, hyper, b1, b2, eps, norm_slots, max_norm, world); break;
    default: dp_adamw_ag_kernel<0><<<grid, 256, 0, s>>>(gshard, w32, m, v, wp, shard, tab, nb, hyper, b1, b2, eps, norm_slots, max_norm, world);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Copy-engine copy between two device addresses (either may be a peer's IPC-mapped buffer) on `s`.
int pcb_memcpy_d2d(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s) == cudaSuccess ? 0 : -3;
}
