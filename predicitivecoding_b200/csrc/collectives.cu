// Peer-memory collectives over NVLink / NVSwitch: all-reduce (one-shot and two-shot),
// reduce-scatter, all-gather and broadcast with Sum / Prod / Max / Min, fp32 or bf16 payloads.
//
// Reference counterpart: PredictiveCoding.Device/Nccl/NcclProvider.cs:1-109, whose four
// collectives run on the host over per-rank float[] buffers.  Here every rank's input sits in a
// symmetric buffer (same size on every rank, mapped into every peer through CUDA IPC), and each
// kernel reads its peers' buffers with plain vectorised loads; the caller brackets the kernel
// with the bounded device barrier so no rank reads a buffer a peer is still writing, and no rank
// reuses its buffer while a peer may still be reading it.  The reduction order over ranks is the
// fixed order 0..world-1 on every rank, so all ranks compute bit-identical results.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "common.cuh"

namespace {

enum : int { kOpSum = 0, kOpProd = 1, kOpMax = 2, kOpMin = 3 };

template <int OP>
__device__ __forceinline__ float combine(float a, float b) {
  if constexpr (OP == kOpSum) return a + b;
  if constexpr (OP == kOpProd) return a * b;
  if constexpr (OP == kOpMax) return fmaxf(a, b);
  return fminf(a, b);
}

template <typename T>
struct Vec;  // 16-byte vector of T
template <>
struct Vec<float> {
  static constexpr int N = 4;
  float v[4];
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __nv_bfloat16 v[8];
};

template <typename T>
__device__ __forceinline__ float to_f(T x) {
  if constexpr (sizeof(T) == 4) return x;
  else return __bfloat162float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x) {
  if constexpr (sizeof(T) == 4) return x;
  else return __float2bfloat16(x);
}

// r[i] = scale * op_{p=0..world-1} in_peers[p][i] for i in [lo, hi), written to out[i - lo] or, with
// out_peers, to out_peers[q][i] of every rank q (the two-shot all-reduce pushes its reduced shard into
// every rank's buffer at the shard's own offsets; each index is read and then overwritten by the same
// thread, and no other rank touches this shard). WORLD > 0 fixes the rank count so that the loads of
// all ranks are issued before the first combine; WORLD == 0 takes it at run time.
template <typename T, int OP, int WORLD>
__global__ void __launch_bounds__(256)
coll_reduce_kernel(const T* const* __restrict__ in_peers, T* __restrict__ out, T* const* __restrict__ out_peers,
                   long long lo, long long hi, int world_rt, float scale) {
  using V = Vec<T>;
  constexpr int N = V::N;
  const int world = WORLD > 0 ? WORLD : world_rt;
  const long long n = hi - lo;
  const bool out_al = out_peers != nullptr || reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const long long nv = (out_al && lo % N == 0) ? n / N : 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nv; q += stride) {
    float acc[N];
    const long long i = lo + q * N;
    if constexpr (WORLD > 0) {
      V x[WORLD];
#pragma unroll
      for (int p = 0; p < WORLD; ++p) x[p] = *reinterpret_cast<const V*>(in_peers[p] + i);
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] = to_f(x[0].v[e]);
#pragma unroll
      for (int p = 1; p < WORLD; ++p)
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] = combine<OP>(acc[e], to_f(x[p].v[e]));
    } else {
      V x = *reinterpret_cast<const V*>(in_peers[0] + i);
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] = to_f(x.v[e]);
#pragma unroll 4
      for (int p = 1; p < world; ++p) {
        V y = *reinterpret_cast<const V*>(in_peers[p] + i);
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] = combine<OP>(acc[e], to_f(y.v[e]));
      }
    }
    V o;
#pragma unroll
    for (int e = 0; e < N; ++e) o.v[e] = from_f<T>(acc[e] * scale);
    if (out_peers != nullptr) {
#pragma unroll 8
      for (int p = 0; p < world; ++p) *reinterpret_cast<V*>(out_peers[p] + i) = o;
    } else {
      *reinterpret_cast<V*>(out + q * N) = o;
    }
  }
  for (long long j = nv * N + blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n; j += stride) {
    float a = to_f(in_peers[0][lo + j]);
    for (int p = 1; p < world; ++p) a = combine<OP>(a, to_f(in_peers[p][lo + j]));
    const T r = from_f<T>(a * scale);
    if (out_peers != nullptr) {
      for (int p = 0; p < world; ++p) out_peers[p][lo + j] = r;
    } else {
      out[j] = r;
    }
  }
}

// out[j * chunk + i] = src_peers[j][j * src_stride + i], i < chunk, j < world  (gather)
// with world == 1 and src_peers = {root buffer} it is a broadcast copy.
template <typename T>
__global__ void __launch_bounds__(256)
coll_gather_kernel(const T* const* __restrict__ src_peers, T* __restrict__ out, long long chunk,
                   long long src_stride, int world) {
  using V = Vec<T>;
  constexpr int N = V::N;
  const bool vec = chunk % N == 0 && src_stride % N == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const long long per = vec ? chunk / N : chunk;
  const long long total = per * world;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < total; q += stride) {
    const int j = static_cast<int>(q / per);
    const long long i = q % per;
    if (vec) {
      *reinterpret_cast<V*>(out + j * chunk + i * N) =
          *reinterpret_cast<const V*>(src_peers[j] + j * src_stride + i * N);
    } else {
      out[j * chunk + i] = src_peers[j][j * src_stride + i];
    }
  }
}

int grid_for(long long work, int num_sms) {
  long long g = (work + 255) / 256;
  const long long cap = (long long)num_sms * 4;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

template <typename T, int OP>
void launch_reduce_op(int g, cudaStream_t s, const T* const* ip, T* o, T* const* op_peers, long long lo, long long hi,
                      int world, float scale) {
  switch (world) {
    case 1: coll_reduce_kernel<T, OP, 1><<<g, 256, 0, s>>>(ip, o, op_peers, lo, hi, world, scale); break;
    case 2: coll_reduce_kernel<T, OP, 2><<<g, 256, 0, s>>>(ip, o, op_peers, lo, hi, world, scale); break;
    case 4: coll_reduce_kernel<T, OP, 4><<<g, 256, 0, s>>>(ip, o, op_peers, lo, hi, world, scale); break;
    case 8: coll_reduce_kernel<T, OP, 8><<<g, 256, 0, s>>>(ip, o, op_peers, lo, hi, world, scale); break;
    default: coll_reduce_kernel<T, OP, 0><<<g, 256, 0, s>>>(ip, o, op_peers, lo, hi, world, scale); break;
  }
}

template <typename T>
int launch_reduce(const void* const* in_peers, void* out, void* const* out_peers, long long lo, long long hi,
                  int world, int op, float scale, int num_sms, cudaStream_t s) {
  auto ip = reinterpret_cast<const T* const*>(in_peers);
  auto o = reinterpret_cast<T*>(out);
  auto opp = reinterpret_cast<T* const*>(out_peers);
  const int g = grid_for((hi - lo) / Vec<T>::N + 1, num_sms);
  switch (op) {
    case kOpSum: launch_reduce_op<T, kOpSum>(g, s, ip, o, opp, lo, hi, world, scale); break;
    case kOpProd: launch_reduce_op<T, kOpProd>(g, s, ip, o, opp, lo, hi, world, scale); break;
    case kOpMax: launch_reduce_op<T, kOpMax>(g, s, ip, o, opp, lo, hi, world, scale); break;
    case kOpMin: launch_reduce_op<T, kOpMin>(g, s, ip, o, opp, lo, hi, world, scale); break;
    default: return -2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace

// dtype: 0 = fp32, 1 = bf16.  in_peers is a device table of world pointers (element type dtype).
int pcb_coll_reduce(const void* const* in_peers, void* out, long long lo, long long hi, int world, int op,
                    float scale, int dtype, int num_sms, cudaStream_t s) {
  if (hi < lo || world < 1) return -2;
  if (hi == lo) return 0;
  return dtype == 0 ? launch_reduce<float>(in_peers, out, nullptr, lo, hi, world, op, scale, num_sms, s)
                    : launch_reduce<__nv_bfloat16>(in_peers, out, nullptr, lo, hi, world, op, scale, num_sms, s);
}

// Reduce [lo, hi) over the ranks' buffers and store the result into every rank's buffer (out_peers) at
// the same offsets: the reduce-scatter and the all-gather halves of a two-shot all-reduce in one pass,
// with the all-gather as pushes (peer stores) rather than pulls.
int pcb_coll_reduce_push(const void* const* in_peers, void* const* out_peers, long long lo, long long hi, int world,
                         int op, float scale, int dtype, int num_sms, cudaStream_t s) {
  if (hi < lo || world < 1 || out_peers == nullptr) return -2;
  if (hi == lo) return 0;
  return dtype == 0 ? launch_reduce<float>(in_peers, nullptr, out_peers, lo, hi, world, op, scale, num_sms, s)
                    : launch_reduce<__nv_bfloat16>(in_peers, nullptr, out_peers, lo, hi, world, op, scale, num_sms, s);
}

int pcb_coll_gather(const void* const* src_peers, void* out, long long chunk, long long src_stride, int world,
                    int dtype, int num_sms, cudaStream_t s) {
  if (chunk <= 0 || world < 1) return chunk == 0 ? 0 : -2;
  const int g = grid_for(chunk * world / 4 + 1, num_sms);
  if (dtype == 0)
    coll_gather_kernel<float><<<g, 256, 0, s>>>(reinterpret_cast<const float* const*>(src_peers),
                                                 reinterpret_cast<float*>(out), chunk, src_stride, world);
  else
    coll_gather_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16* const*>(src_peers),
                                                         reinterpret_cast<__nv_bfloat16*>(out), chunk, src_stride,
                                                         world);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
