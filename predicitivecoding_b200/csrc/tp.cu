// Tensor-parallel helpers: the owner side of the fused GEMM -> reduce-scatter.
//
// A row-parallel GEMM (EPI_RS_BF16) leaves, on every owner rank, world partial blocks
// slots[s] = (rank s's partial product for this owner's rows), bf16 [world, rows, D].  This
// kernel sums them in fp32 in rank order (deterministic), adds the residual stream, stores the new
// residual, and -- sequence-parallel RMSNorm -- writes the normalised row in bf16 straight into this
// rank's chunk of the next all-gather buffer, together with 1/rms for the backward.
// The reference has no tensor parallelism on a GPU (PredictiveCoding.LLM/Infrastructure/
// TensorParallel.cs:20-141 splits single matvecs over CPU tasks).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"

using namespace pcb;

namespace {

constexpr int kTpThreads = 256;

// x_out[r] = resid[r] + sum_s slots[s][r]   (resid may be nullptr: plain reduction)
// if gamma: y[r] = x_out[r] * gamma / rms(x_out[r]) (bf16, row stride ldy), inv[r] = 1/rms
__global__ void __launch_bounds__(kTpThreads)
tp_reduce_norm_kernel(const __nv_bfloat16* __restrict__ slots, int world, int rows, int D,
                      const float* __restrict__ resid, float* __restrict__ x_out, int accumulate,
                      const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ y, long long ldy,
                      float* __restrict__ inv, float eps) {
  const int r = blockIdx.x;
  const long long slot_stride = (long long)rows * D;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < D; i += kTpThreads * 8) {
    float acc[8];
    const long long o = (long long)r * D + i;
    if (resid != nullptr) {
      const float4 a = *reinterpret_cast<const float4*>(resid + o);
      const float4 b = *reinterpret_cast<const float4*>(resid + o + 4);
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
      acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
    } else if (accumulate) {
      const float4 a = *reinterpret_cast<const float4*>(x_out + o);
      const float4 b = *reinterpret_cast<const float4*>(x_out + o + 4);
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
      acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    }
    for (int s = 0; s < world; ++s) {
      const uint4 u = *reinterpret_cast<const uint4*>(slots + s * slot_stride + o);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    *reinterpret_cast<float4*>(x_out + o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(x_out + o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += acc[e] * acc[e];
  }
  if (gamma == nullptr) return;
  __shared__ float red[kTpThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kTpThreads / 32; ++w) tot += red[w];
  const float rinv = rsqrtf(tot / D + eps);
  if (threadIdx.x == 0) inv[r] = rinv;
  for (int i = threadIdx.x * 8; i < D; i += kTpThreads * 8) {
    const long long o = (long long)r * D + i;
    const float4 a = *reinterpret_cast<const float4*>(x_out + o);
    const float4 b = *reinterpret_cast<const float4*>(x_out + o + 4);
    const uint4 gu = *reinterpret_cast<const uint4*>(gamma + i);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gu);
    const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint4 out;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = __bfloat1622float2(g2[e]);
      ow[e] = pack_bf16x2(xv[2 * e] * rinv * g.x, xv[2 * e + 1] * rinv * g.y);
    }
    *reinterpret_cast<uint4*>(y + (long long)r * ldy + i) = out;
  }
}

}  // namespace

int pcb_tp_reduce_norm(const void* slots, int world, int rows, int D, const float* resid, float* x_out,
                       int accumulate, const void* gamma, void* y, long long ldy, float* inv, float eps,
                       cudaStream_t s) {
  if (D % 8 || rows <= 0 || world <= 0) return -2;
  tp_reduce_norm_kernel<<<rows, kTpThreads, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(slots), world, rows, D,
                                                      resid, x_out, accumulate,
                                                      reinterpret_cast<const __nv_bfloat16*>(gamma),
                                                      reinterpret_cast<__nv_bfloat16*>(y), ldy, inv, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

namespace {
// x[r] += sum_s peers[s][r] (bf16 partial products read from every rank's buffer over NVLink, summed
// in rank order), then y[r] = x[r] * gamma / rms(x[r]) in bf16: the all-reduce of a row-parallel
// product fused with the residual add and the next RMSNorm.  Rows are replicated on every rank.
//
// With `flags` (sync variant) the kernel also replaces the device barrier that must precede it: CTA r
// (row r) bumps its own epoch counter ctr[r], stores it into slot [r][rank] of every rank's flag array
// (release, system scope) and waits until slot [r][p] of its own array holds that epoch for every p
// (acquire; bounded, error code on timeout).  A peer reaches the store only after its row-parallel
// product (the kernel before it in its stream) has completed, and each row only reads row r of the
// peers' partials, so a per-row handshake is all the ordering the reads need; the partial buffers are
// double-buffered, so a buffer is rewritten only after every rank has passed the next handshake.
__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kTpThreads)
tp_allreduce_norm_kernel(const __nv_bfloat16* const* __restrict__ peers, int world, int D, float* __restrict__ x,
                         const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ y, float eps,
                         unsigned int* const* __restrict__ flags, unsigned int* __restrict__ ctr, int rank,
                         int* __restrict__ err) {
  pdl_begin();
  const int r = blockIdx.x;
  if (flags != nullptr) {
    __shared__ unsigned int epoch;
    if (threadIdx.x == 0) {
      epoch = ctr[r] + 1;
      ctr[r] = epoch;
    }
    __syncthreads();
    const unsigned int e = epoch;
    const int p = threadIdx.x;
    if (p < world) {
      st_release_sys_u32(flags[p] + (long long)r * world + rank, e);
      const unsigned int* mine = flags[rank] + (long long)r * world + p;
      const long long t0 = clock64();
      while (ld_acquire_sys_u32(mine) < e) {
        if (clock64() - t0 > kSpinBudgetCycles) {
          record_error(err, kErrTimeoutPeer);
          break;
        }
      }
    }
    __syncthreads();
  }
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < D; i += kTpThreads * 8) {
    const long long o = (long long)r * D + i;
    const float4 a = *reinterpret_cast<const float4*>(x + o);
    const float4 b = *reinterpret_cast<const float4*>(x + o + 4);
    float acc[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    for (int s = 0; s < world; ++s) {
      const uint4 u = *reinterpret_cast<const uint4*>(peers[s] + o);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    *reinterpret_cast<float4*>(x + o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(x + o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += acc[e] * acc[e];
  }
  __shared__ float red[kTpThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kTpThreads / 32; ++w) tot += red[w];
  const float rinv = rsqrtf(tot / D + eps);
  for (int i = threadIdx.x * 8; i < D; i += kTpThreads * 8) {
    const long long o = (long long)r * D + i;
    const float4 a = *reinterpret_cast<const float4*>(x + o);
    const float4 b = *reinterpret_cast<const float4*>(x + o + 4);
    const uint4 gu = *reinterpret_cast<const uint4*>(gamma + i);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gu);
    const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint4 out;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = __bfloat1622float2(g2[e]);
      ow[e] = pack_bf16x2(xv[2 * e] * rinv * g.x, xv[2 * e + 1] * rinv * g.y);
    }
    *reinterpret_cast<uint4*>(y + o) = out;
  }
}
}  // namespace

// peers: device array of `world` pointers to [rows, D] bf16 partials (this rank's included).  Without
// `flags` the caller orders it after a barrier that follows every rank's write of its partial; with
// `flags` (device array of `world` pointers to [rows, world] uint32 flag arrays, one per rank, zero at
// first) and `ctr` ([rows] uint32 epochs, this rank's) the kernel does the per-row handshake itself.
int pcb_tp_allreduce_norm(const void* peers, int world, int rows, int D, float* x, const void* gamma, void* y,
                          float eps, void* const* flags, unsigned int* ctr, int rank, int* err, cudaStream_t s) {
  if (D % 8 || rows <= 0 || world <= 0 || world > kTpThreads) return -2;
  if (flags != nullptr && ctr == nullptr) return -2;
  pdl_launch(tp_allreduce_norm_kernel, dim3(rows), dim3(kTpThreads), 0, s,
             reinterpret_cast<const __nv_bfloat16* const*>(peers), world, D, x,
             reinterpret_cast<const __nv_bfloat16*>(gamma), reinterpret_cast<__nv_bfloat16*>(y), eps,
             reinterpret_cast<unsigned int* const*>(flags), ctr, rank, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
