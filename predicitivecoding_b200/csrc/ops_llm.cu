// Bandwidth-bound kernels of the decoder training step (sm_100a).
//
// Reference kernels these replace (PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs):
//   embed_gather :37-42, embed_scatter :50-55, col_sum_acc :82-92, rms_fwd :154-173,
//   rms_bwd_dx :182-203, rms_dgamma :212-223, rope_s :237-254, ce_loss_grad :503-537,
//   adam_step :584-598.  The reference runs one launch per parameter tensor for AdamW;
//   here the whole parameter arena is one flat buffer and one launch updates it.
#include <cstdint>

#include "common.cuh"

namespace pcb {

// ------------------------------------------------------------------ embedding
// x[t,:] = W[tok[t],:]   (fp32 residual stream)
// W is the bf16 working copy of the table (the fp32 master may be sharded across ranks).
// Checked builds (-DPCB_CHECKED, setup.py with PCB_CHECKED=1) count the out-of-range token ids that the
// embedding kernels clamp or skip, so a test can assert that none occurred.
#ifdef PCB_CHECKED
__device__ unsigned long long g_checked_violations = 0;
#define PCB_COUNT_VIOLATION() atomicAdd(&g_checked_violations, 1ull)
#else
#define PCB_COUNT_VIOLATION() ((void)0)
#endif

__global__ void embed_fwd_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ W,
                                 float* __restrict__ x, int M, int D, int V) {
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= M) return;
  int id = tok[t];
  if ((id < 0 || id >= V) && threadIdx.x == 0) PCB_COUNT_VIOLATION();
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const uint2* src = reinterpret_cast<const uint2*>(W + (long long)id * D);
  float4* dst = reinterpret_cast<float4*>(x + (long long)t * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
    const uint2 u = src[i];
    dst[i] = make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
  }
}

// dW[tok[t],:] += dx[t,:]
__global__ void embed_bwd_kernel(const int* __restrict__ tok, const float* __restrict__ dx, float* __restrict__ dW,
                                 int M, int D, int V) {
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= M) return;
  int id = tok[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) PCB_COUNT_VIOLATION();
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(dx + (long long)t * D);
  float4* dst = reinterpret_cast<float4*>(dW + (long long)id * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) atomicAdd(dst + i, src[i]);
}

// ------------------------------------------------------------------ RMSNorm
PCB_DEVICE float4 load_g4(const __nv_bfloat16* g, int c) {
  const uint2 u = reinterpret_cast<const uint2*>(g)[c];
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
}
// y = x * g * inv,  inv = 1/sqrt(mean(x^2) + eps).  One warp per row.
// Reference: PredictiveCoding.LLM/Autograd/Autograd.cs:435-472.
template <int VPT>  // float4 vectors per lane
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ g,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ inv_out, int M, int D,
                                   float eps) {
  pdl_wait();
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * D);
  float4 v[VPT];
  float ss = 0.f;
  const int nvec = D / 4;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      v[i] = xr[c];
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  if (lane == 0 && inv_out) inv_out[row] = inv;
  uint2* yr = reinterpret_cast<uint2*>(y + (long long)row * D);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      const float4 gg = load_g4(g, c);
      uint2 o;
      o.x = pack_bf16x2(v[i].x * inv * gg.x, v[i].y * inv * gg.y);
      o.y = pack_bf16x2(v[i].z * inv * gg.z, v[i].w * inv * gg.w);
      yr[c] = o;
    }
  }
}

// dx (+)= inv * (g*dy - x * inv^2 * mean(g*dy*x)) ; dg += dy * x * inv   (dy fp32)
template <int VPT>
__global__ void rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ g, const float* __restrict__ inv_in,
                                   float* __restrict__ dx, __nv_bfloat16* __restrict__ dx16, float* __restrict__ dg,
                                   int M, int D, int accumulate) {
  pdl_wait();
  extern __shared__ float sdg[];  // [D] per-block dgamma partial
  for (int i = threadIdx.x; i < D; i += blockDim.x) sdg[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = D / 4;
  float4 dga[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) dga[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += gridDim.x * warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * D);
    const float4* dyr = reinterpret_cast<const float4*>(dy + (long long)row * D);
    float4* dxr = reinterpret_cast<float4*>(dx + (long long)row * D);
    const float inv = inv_in[row];
    // Up to D = 1024 every load of the row (x, dy and, when accumulating, dx) is issued before any
    // arithmetic; wider rows read the previous dx at the store, which keeps the row within registers.
    constexpr bool kBatchPrev = VPT <= 8;
    constexpr int PV = kBatchPrev ? VPT : 1;
    float4 xv[VPT], dv[VPT], pv[PV];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        xv[i] = xr[c];
        dv[i] = dyr[c];
        if constexpr (kBatchPrev) pv[i] = accumulate ? dxr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 gg = load_g4(g, c);
        dot += gg.x * dv[i].x * xv[i].x + gg.y * dv[i].y * xv[i].y + gg.z * dv[i].z * xv[i].z +
               gg.w * dv[i].w * xv[i].w;
        dga[i].x += dv[i].x * xv[i].x * inv;
        dga[i].y += dv[i].y * xv[i].y * inv;
        dga[i].z += dv[i].z * xv[i].z * inv;
        dga[i].w += dv[i].w * xv[i].w * inv;
      }
    }
    dot = warp_sum(dot);
    const float k = inv * inv * dot / (float)D;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        const float4 gg = load_g4(g, c);
        float4 p;
        if constexpr (kBatchPrev) p = pv[i];
        else p = accumulate ? dxr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 o;
        o.x = inv * (gg.x * dv[i].x - xv[i].x * k) + p.x;
        o.y = inv * (gg.y * dv[i].y - xv[i].y * k) + p.y;
        o.z = inv * (gg.z * dv[i].z - xv[i].z * k) + p.z;
        o.w = inv * (gg.w * dv[i].w - xv[i].w * k) + p.w;
        dxr[c] = o;
        if (dx16 != nullptr) {
          uint2 u;
          u.x = pack_bf16x2(o.x, o.y);
          u.y = pack_bf16x2(o.z, o.w);
          reinterpret_cast<uint2*>(dx16 + (long long)row * D)[c] = u;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      atomicAdd(&sdg[4 * c + 0], dga[i].x);
      atomicAdd(&sdg[4 * c + 1], dga[i].y);
      atomicAdd(&sdg[4 * c + 2], dga[i].z);
      atomicAdd(&sdg[4 * c + 3], dga[i].w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) atomicAdd(&dg[i], sdg[i]);
}

// ------------------------------------------------------------------ RoPE
// Interleaved pairs (2i, 2i+1) per head, angle = pos * 10000^(-2i/hd), pos = row % S.
// Applied in place to the first `nparts` D-wide parts of a [M, ld] bf16 buffer
// (q and k of the fused qkv activations).  sign = -1 rotates backwards (gradients).
// Reference: PredictiveCoding.LLM/Autograd/Autograd.cs:475-508, DeviceTrainKernels.cs:237-254.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ buf, long long ld, const float2* __restrict__ cs,
                            int M, int S, int D, int hd, int nparts, float sign) {
  const int half = hd / 2;
  const long long pairs_per_row = (long long)nparts * (D / 2);
  const long long total = (long long)M * pairs_per_row;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(idx / pairs_per_row);
    const int p = (int)(idx % pairs_per_row);
    const int part = p / (D / 2);
    const int q = p % (D / 2);
    const int i = q % half;  // pair index within head
    const int pos = row % S;
    const float2 c = cs[pos * half + i];
    __nv_bfloat162* ptr = reinterpret_cast<__nv_bfloat162*>(buf + row * ld + (long long)part * D) + q;
    const float2 v = __bfloat1622float2(*ptr);
    const float sn = sign * c.y;
    *ptr = __floats2bfloat162_rn(v.x * c.x - v.y * sn, v.x * sn + v.y * c.x);
  }
}

// ------------------------------------------------------------------ cross-entropy
// loss[r] = lse(logits[r]) - logits[r, t];  dlogits[r] = (softmax - onehot) * scale, in place (bf16).
// targets < 0 are ignored (zero loss and zero gradient).  Reference (device path, pure LSE):
// PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs:503-537.
__global__ void ce_fwd_bwd_kernel(__nv_bfloat16* __restrict__ logits, long long ld, const int* __restrict__ tgt,
                                  float* __restrict__ loss, int M, int V, float scale, int write_grad) {
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= M) return;
  __nv_bfloat16* row = logits + (long long)r * ld;
  const int t = tgt[r];
  __shared__ float s_m[32], s_s[32];
  float mx = -INFINITY, sm = 0.f;
  // 16-byte vectors when the row stride allows them; the rest is handled element-wise
  const int nvec = (ld % 8 == 0 && ((uintptr_t)logits & 15) == 0) ? V / 8 : 0;
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const uint4 u = rv[i];
    float f[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                  bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    if (lm > mx) {
      sm *= __expf(mx - lm);
      mx = lm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sm += __expf(f[j] - mx);
  }
  for (int j = 8 * nvec + threadIdx.x; j < V; j += blockDim.x) {
    const float f = __bfloat162float(row[j]);
    if (f > mx) {
      sm = (mx == -INFINITY ? 0.f : sm * __expf(mx - f));
      mx = f;
    }
    sm += __expf(f - mx);
  }
  // combine (max, sum) pairs across the block
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const float os = __shfl_xor_sync(0xffffffffu, sm, o);
    const float nm = fmaxf(mx, om);
    sm = (mx == -INFINITY ? 0.f : sm * __expf(mx - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    mx = nm;
  }
  if (lane == 0) { s_m[w] = mx; s_s[w] = sm; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    mx = lane < nw ? s_m[lane] : -INFINITY;
    sm = lane < nw ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const float os = __shfl_xor_sync(0xffffffffu, sm, o);
      const float nm = fmaxf(mx, om);
      sm = (mx == -INFINITY ? 0.f : sm * __expf(mx - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      mx = nm;
    }
    if (lane == 0) { s_m[0] = mx; s_s[0] = sm; }
  }
  __syncthreads();
  mx = s_m[0];
  const float lse = mx + __logf(s_s[0]);
  if (threadIdx.x == 0) {
    loss[r] = (t >= 0 && t < V) ? lse - __bfloat162float(row[t]) : 0.f;
  }
  if (!write_grad) return;
  __syncthreads();  // the target logit is read above before being overwritten below
  uint4* wv = reinterpret_cast<uint4*>(row);
  const bool counted = (t >= 0 && t < V);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const uint4 u = wv[i];
    float f[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                  bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p = counted ? __expf(f[j] - lse) : 0.f;
      if (counted && 8 * i + j == t) p -= 1.f;
      f[j] = p * scale;
    }
    uint4 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    o.z = pack_bf16x2(f[4], f[5]);
    o.w = pack_bf16x2(f[6], f[7]);
    wv[i] = o;
  }
  for (int j = 8 * nvec + threadIdx.x; j < V; j += blockDim.x) {
    float p = counted ? __expf(__bfloat162float(row[j]) - lse) : 0.f;
    if (counted && j == t) p -= 1.f;
    row[j] = __float2bfloat16(p * scale);
  }
}

// Register-resident variant for V <= 8 * 512 * RV (V % 8 == 0): a persistent block of 512 threads owns
// one row at a time with the whole row in registers, so each logit is read once, exponentiated once
// (p = exp(f - max) is kept for the gradient) and written once.  The next row's loads are issued
// before the block-wide sum reduction of the current row, so HBM traffic continues through the
// reductions and the gradient stores.
template <int RV>
__global__ void __launch_bounds__(512, 1)
    ce_rows_kernel(__nv_bfloat16* __restrict__ logits, long long ld, const int* __restrict__ tgt,
                   float* __restrict__ loss, int M, int V, float scale, int write_grad) {
  pdl_wait();
  __shared__ float red_m[2][16], red_s[2][16];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nvec = V >> 3;
  int r = blockIdx.x;
  if (r >= M) return;
  uint4 raw[RV];
  auto load_row = [&](int row) {
    const uint4* rv = reinterpret_cast<const uint4*>(logits + (long long)row * ld);
#pragma unroll
    for (int i = 0; i < RV; ++i) {
      const int c = tid + 512 * i;
      raw[i] = c < nvec ? rv[c] : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);  // -inf
    }
  };
  load_row(r);
  int par = 0;
  while (true) {
    const int t = tgt[r];
    const bool counted = t >= 0 && t < V;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < RV; ++i) {
      mx = fmaxf(mx, fmaxf(fmaxf(bf16_lo(raw[i].x), bf16_hi(raw[i].x)), fmaxf(bf16_lo(raw[i].y), bf16_hi(raw[i].y))));
      mx = fmaxf(mx, fmaxf(fmaxf(bf16_lo(raw[i].z), bf16_hi(raw[i].z)), fmaxf(bf16_lo(raw[i].w), bf16_hi(raw[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red_m[par][w] = mx;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) mx = fmaxf(mx, red_m[par][k]);
    float p[RV * 8];
    float sm = 0.f, ft = 0.f;
    bool own = false;
#pragma unroll
    for (int i = 0; i < RV; ++i) {
      const float f[8] = {bf16_lo(raw[i].x), bf16_hi(raw[i].x), bf16_lo(raw[i].y), bf16_hi(raw[i].y),
                          bf16_lo(raw[i].z), bf16_hi(raw[i].z), bf16_lo(raw[i].w), bf16_hi(raw[i].w)};
      const int base = 8 * (tid + 512 * i);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        p[8 * i + j] = __expf(f[j] - mx);
        sm += p[8 * i + j];
        if (base + j == t) { ft = f[j]; own = true; }
      }
    }
    const int next = r + gridDim.x;
    if (next < M) load_row(next);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane == 0) red_s[par][w] = sm;
    __syncthreads();
    sm = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) sm += red_s[par][k];
    if (own) loss[r] = mx + __logf(sm) - ft;
    else if (!counted && tid == 0) loss[r] = 0.f;
    if (write_grad) {
      const float k = counted ? scale / sm : 0.f;
      uint4* wv = reinterpret_cast<uint4*>(logits + (long long)r * ld);
#pragma unroll
      for (int i = 0; i < RV; ++i) {
        const int c = tid + 512 * i;
        if (c < nvec) {
          float g[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) g[j] = p[8 * i + j] * k - (8 * c + j == t ? scale : 0.f);
          uint4 o;
          o.x = pack_bf16x2(g[0], g[1]);
          o.y = pack_bf16x2(g[2], g[3]);
          o.z = pack_bf16x2(g[4], g[5]);
          o.w = pack_bf16x2(g[6], g[7]);
          wv[c] = o;
        }
      }
    }
    if (next >= M) break;
    r = next;
    par ^= 1;
  }
}

// ------------------------------------------------------------------ reductions
// out[0] += sum(x^2) over n elements (global-norm clipping).
__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ out, int square) {
  pdl_wait();
  float s = 0.f;
  const long long n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = x4[i];
    // NaN/Inf gradients count as zero (reference GradientClipping zeroes them,
    // PredictiveCoding.LLM/Training/Optimizers.cs:100-104)
    if (square)
      s += (isfinite(v.x) ? v.x * v.x : 0.f) + (isfinite(v.y) ? v.y * v.y : 0.f) +
           (isfinite(v.z) ? v.z * v.z : 0.f) + (isfinite(v.w) ? v.w * v.w : 0.f);
    else
      s += v.x + v.y + v.z + v.w;
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    s += square ? (isfinite(x[i]) ? x[i] * x[i] : 0.f) : x[i];
  s = warp_sum(s);
  __shared__ float sh[32];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) atomicAdd(out, s);
  }
}

PCB_DEVICE float to_f(float v) { return v; }
PCB_DEVICE float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// out[n] (+)= sum over rows of x[m, n]   (bf16 or fp32 input)
template <typename T>
__global__ void colsum_kernel(const T* __restrict__ x, long long ld, float* __restrict__ out, int M, int N, float scale) {
  pdl_wait();
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int rows_per = (M + gridDim.y - 1) / gridDim.y;
  const int r0 = blockIdx.y * rows_per, r1 = min(M, r0 + rows_per);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += to_f(x[(long long)r * ld + n]);
  atomicAdd(out + n, s * scale);
}

// ------------------------------------------------------------------ AdamW
// Decoupled decay applied AFTER the Adam step, on the updated weight (reference order,
// PredictiveCoding.LLM/Training/Optimizers.cs:50-54 and DeviceTrainKernels.cs:593-597):
//   w -= lr * mhat / (sqrt(vhat) + eps);  w -= lr * wd * w
// grad_scale folds the micro-batch mean; clip (if non-null) holds sum(g^2) and the
// gradient is further scaled by min(1, max_norm / ||g||).  Non-finite grads count as 0.
// wd applies to elements [0, n_decay); elements beyond it are not decayed.
// hyper = [lr, wd, bc1, bc2, grad_scale] lives in device memory so a captured CUDA graph
// replays the optimizer with the current schedule values.
PCB_DEVICE void adamw_elem(float& wi, float gi, float& mi, float& vi, long long i, long long n_decay, float s,
                           float lr, float wd, float bc1, float bc2, float b1, float b2, float eps) {
  gi = isfinite(gi) ? gi * s : 0.f;
  mi = b1 * mi + (1.f - b1) * gi;
  vi = b2 * vi + (1.f - b2) * gi * gi;
  wi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
  if (i < n_decay) wi -= lr * wd * wi;
}

// Four parameters per thread and step (16-byte loads of w, g, m, v; 8-byte bf16 store), two such
// groups in flight per thread; the n % 4 tail (or an unaligned buffer) takes the scalar loop.
__global__ void adamw_kernel(float* __restrict__ w, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ w16, long long n,
                             long long n_decay, const float* __restrict__ hyper, float b1, float b2, float eps,
                             const float* __restrict__ clip_sumsq, float max_norm) {
  pdl_wait();
  const float lr = hyper[0], wd = hyper[1], bc1 = hyper[2], bc2 = hyper[3];
  float s = hyper[4];
  const float grad_scale = s;
  if (clip_sumsq != nullptr && max_norm > 0.f) {
    const float norm = sqrtf(*clip_sumsq) * grad_scale;
    if (norm > max_norm) s *= max_norm / (norm + 1e-6f);
  }
  const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
                     reinterpret_cast<uintptr_t>(v)) & 15) == 0 &&
                   (w16 == nullptr || (reinterpret_cast<uintptr_t>(w16) & 7) == 0);
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long done = 0;
  if (vec) {
    const long long n4 = n / 4;
    float4* w4 = reinterpret_cast<float4*>(w);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    float4* m4 = reinterpret_cast<float4*>(m);
    float4* v4 = reinterpret_cast<float4*>(v);
    for (long long i = tid; i < n4; i += 2 * stride) {
      const long long j = i + stride;
      const bool two = j < n4;
      float4 wa = w4[i], ga = g4[i], ma = m4[i], va = v4[i];
      float4 wb, gb, mb, vb;
      if (two) { wb = w4[j]; gb = g4[j]; mb = m4[j]; vb = v4[j]; }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1 && !two) break;
        const long long q = h ? j : i;
        float4& wq = h ? wb : wa;
        float4& gq = h ? gb : ga;
        float4& mq = h ? mb : ma;
        float4& vq = h ? vb : va;
        adamw_elem(wq.x, gq.x, mq.x, vq.x, 4 * q + 0, n_decay, s, lr, wd, bc1, bc2, b1, b2, eps);
        adamw_elem(wq.y, gq.y, mq.y, vq.y, 4 * q + 1, n_decay, s, lr, wd, bc1, bc2, b1, b2, eps);
        adamw_elem(wq.z, gq.z, mq.z, vq.z, 4 * q + 2, n_decay, s, lr, wd, bc1, bc2, b1, b2, eps);
        adamw_elem(wq.w, gq.w, mq.w, vq.w, 4 * q + 3, n_decay, s, lr, wd, bc1, bc2, b1, b2, eps);
        m4[q] = mq;
        v4[q] = vq;
        w4[q] = wq;
        if (w16 != nullptr)
          reinterpret_cast<uint2*>(w16)[q] = make_uint2(pack_bf16x2(wq.x, wq.y), pack_bf16x2(wq.z, wq.w));
      }
    }
    done = 4 * n4;
  }
  for (long long i = done + tid; i < n; i += stride) {
    float wi = w[i], mi = m[i], vi = v[i];
    adamw_elem(wi, g[i], mi, vi, i, n_decay, s, lr, wd, bc1, bc2, b1, b2, eps);
    m[i] = mi;
    v[i] = vi;
    w[i] = wi;
    if (w16 != nullptr) w16[i] = __float2bfloat16_rn(wi);
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

}  // namespace pcb

using namespace pcb;

// ---------------------------------------------------------------- host launchers
static int grid_for(long long n, int threads, int cap = 148 * 16) {
  long long b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > cap) b = cap;
  return (int)b;
}

int pcb_embed_fwd(const int* tok, const void* W, float* x, int M, int D, int V, cudaStream_t s) {
  if (D % 4) return -1;
  step_launch(embed_fwd_kernel, dim3(M), dim3(128), 0, s, tok, reinterpret_cast<const __nv_bfloat16*>(W), x, M, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Number of bounds violations counted since the last call (and reset it); -1 in unchecked builds.
long long pcb_checked_violations() {
#ifdef PCB_CHECKED
  unsigned long long v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_checked_violations, sizeof(v)) != cudaSuccess) return -2;
  cudaMemcpyToSymbol(g_checked_violations, &zero, sizeof(zero));
  return (long long)v;
#else
  return -1;
#endif
}

int pcb_embed_bwd(const int* tok, const float* dx, float* dW, int M, int D, int V, cudaStream_t s) {
  if (D % 4) return -1;
  step_launch(embed_bwd_kernel, dim3(M), dim3(128), 0, s, tok, dx, dW, M, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_rmsnorm_fwd(const float* x, const void* gv, void* y, float* inv, int M, int D, float eps, cudaStream_t s) {
  if (D % 4 || D > 4096) return -1;
  const int rows_per_block = 8;
  const int grid = (M + rows_per_block - 1) / rows_per_block;
  __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y);
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(gv);
  if (D <= 512) step_launch(rmsnorm_fwd_kernel<4>, dim3(grid), dim3(256), 0, s, x, g, yb, inv, M, D, eps);
  else if (D <= 1024) step_launch(rmsnorm_fwd_kernel<8>, dim3(grid), dim3(256), 0, s, x, g, yb, inv, M, D, eps);
  else if (D <= 2048) step_launch(rmsnorm_fwd_kernel<16>, dim3(grid), dim3(256), 0, s, x, g, yb, inv, M, D, eps);
  else step_launch(rmsnorm_fwd_kernel<32>, dim3(grid), dim3(256), 0, s, x, g, yb, inv, M, D, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// One warp per row with exactly ceil(D / 128) float4 per lane (registers are sized to the row, so
// occupancy is not spent on unused lanes); a persistent grid of every block that fits at once.
template <int VPT>
static int launch_rmsnorm_bwd(const float* dy, const float* x, const __nv_bfloat16* g, const float* inv, float* dx,
                              __nv_bfloat16* dx16, float* dg, int M, int D, int accumulate, int num_sms,
                              cudaStream_t s) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rmsnorm_bwd_kernel<VPT>, 256, 128 * VPT * sizeof(float));
    per_sm = n > 0 ? n : 1;
  }
  int grid = (M + 7) / 8;
  const int cap = (num_sms > 0 ? num_sms : 148) * per_sm;
  if (grid > cap) grid = cap;
  step_launch(rmsnorm_bwd_kernel<VPT>, dim3(grid), dim3(256), (size_t)D * sizeof(float), s, dy, x, g, inv, dx, dx16, dg, M, D, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_rmsnorm_bwd(const float* dy, const float* x, const void* gv, const float* inv, float* dx, void* dx16v,
                    float* dg, int M, int D, int accumulate, int num_sms, cudaStream_t s) {
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(gv);
  __nv_bfloat16* dx16 = reinterpret_cast<__nv_bfloat16*>(dx16v);
  if (D % 4 || D > 4096) return -1;
  if (M <= 0) return 0;
  const int v = (D / 4 + 31) / 32;
#define PCB_RMS_BWD(N) launch_rmsnorm_bwd<N>(dy, x, g, inv, dx, dx16, dg, M, D, accumulate, num_sms, s)
  switch (v) {
    case 1: return PCB_RMS_BWD(1);
    case 2: return PCB_RMS_BWD(2);
    case 3: return PCB_RMS_BWD(3);
    case 4: return PCB_RMS_BWD(4);
    case 5: return PCB_RMS_BWD(5);
    case 6: return PCB_RMS_BWD(6);
    case 7: return PCB_RMS_BWD(7);
    case 8: return PCB_RMS_BWD(8);
    default: break;
  }
  if (v <= 12) return PCB_RMS_BWD(12);
  if (v <= 16) return PCB_RMS_BWD(16);
  if (v <= 24) return PCB_RMS_BWD(24);
  return PCB_RMS_BWD(32);
#undef PCB_RMS_BWD
}

int pcb_rope(void* buf, long long ld, const float* cs, int M, int S, int D, int hd, int nparts, float sign,
             cudaStream_t s) {
  if (hd % 2 || D % hd) return -1;
  const long long total = (long long)M * nparts * (D / 2);
  rope_kernel<<<grid_for(total, 256), 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(buf), ld,
                                                     reinterpret_cast<const float2*>(cs), M, S, D, hd, nparts, sign);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_ce(void* logits, long long ld, const int* tgt, float* loss, int M, int V, float scale, int write_grad,
           cudaStream_t s) {
  if (M <= 0) return 0;
  const int nvec = V / 8;
  if (((uintptr_t)logits & 15) == 0 && ld % 8 == 0 && V % 8 == 0 && nvec <= 8 * 512 && M > 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = M < sms ? M : sms;
    auto* lg = reinterpret_cast<__nv_bfloat16*>(logits);
    if (nvec <= 512) step_launch(ce_rows_kernel<1>, dim3(grid), dim3(512), 0, s, lg, ld, tgt, loss, M, V, scale, write_grad);
    else if (nvec <= 1024) step_launch(ce_rows_kernel<2>, dim3(grid), dim3(512), 0, s, lg, ld, tgt, loss, M, V, scale, write_grad);
    else if (nvec <= 2048) step_launch(ce_rows_kernel<4>, dim3(grid), dim3(512), 0, s, lg, ld, tgt, loss, M, V, scale, write_grad);
    else step_launch(ce_rows_kernel<8>, dim3(grid), dim3(512), 0, s, lg, ld, tgt, loss, M, V, scale, write_grad);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  step_launch(ce_fwd_bwd_kernel, dim3(M), dim3(512), 0, s, reinterpret_cast<__nv_bfloat16*>(logits), ld, tgt, loss, M, V, scale,
                                       write_grad);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_sumsq(const float* x, long long n, float* out, int square, cudaStream_t s) {
  step_launch(sumsq_kernel, dim3(grid_for(n / 4 + 1, 512, 148 * 4)), dim3(512), 0, s, x, n, out, square);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_colsum(const void* x, int is_bf16, long long ld, float* out, int M, int N, float scale, cudaStream_t s) {
  dim3 grid((N + 255) / 256, 64);
  if (is_bf16)
    step_launch(colsum_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(x), ld, out, M, N, scale);
  else
    step_launch(colsum_kernel<float>, dim3(grid), dim3(256), 0, s, reinterpret_cast<const float*>(x), ld, out, M, N, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_adamw(float* w, const float* g, float* m, float* v, void* w16, long long n, long long n_decay,
              const float* hyper, float b1, float b2, float eps, const float* clip_sumsq, float max_norm,
              cudaStream_t s) {
  step_launch(adamw_kernel, dim3(grid_for(n, 256, 148 * 8)), dim3(256), 0, s, w, g, m, v, reinterpret_cast<__nv_bfloat16*>(w16), n,
                                                           n_decay, hyper, b1, b2, eps, clip_sumsq, max_norm);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_f32_to_bf16(const float* x, void* y, long long n, cudaStream_t s) {
  f32_to_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, reinterpret_cast<__nv_bfloat16*>(y), n);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
