// Mixture-of-experts FFN on the device: routing, dispatch into expert-sorted segments, gather,
// combine, and their backward.  The expert FFNs themselves run as grouped tcgen05 GEMMs on the
// CTA-pair kernel (pcb_gemm_grouped_launch).
//
// Reference counterpart: PredictiveCoding.LLM/Autograd/DecoderLM.cs:556-615 -- the router softmax
// over all experts, the top-k experts of every row, a gate-weighted sum of GELU expert FFNs (with
// biases), and the Switch balance loss E * sum_e mean_t(gate[t, e]) * frac_e, frac_e = rows routed to
// e / (rows * k).  The reference loops over experts and runs each on its routed rows; here the
// (token, slot) assignments are sorted by expert once per layer so every expert's rows are one
// contiguous, 256-row-padded segment of a buffer that the grouped GEMM walks tile by tile.
//
// Layout: gates [M, E] fp32 (the full softmax), topi [M, k] int32, pos [M, k] int32 (row of each
// assignment in the sorted buffer), src [cap] int32 (token of each sorted row, -1 for padding),
// rgate [cap] fp32 (gate of each sorted row, 0 for padding), seg [E + 1] int32 (segment starts,
// multiples of 256; seg[E] = rows in use).
#include "common.cuh"

namespace pcb {
namespace moe {

constexpr int kSeg = 256;    // segment alignment: the CTA-pair GEMM's tile rows
constexpr int kMaxE = 64;
constexpr int kMaxK = 8;

PCB_DEVICE void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = bf16_lo(w[j]);
    f[2 * j + 1] = bf16_hi(w[j]);
  }
}

// ---------------------------------------------------------------- routing: one warp per token
template <int MAXE>
__global__ void route_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ router,
                             int M, int D, int E, int k, float* __restrict__ gates, int* __restrict__ topi) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < M; t += warps) {
    float acc[MAXE];
#pragma unroll
    for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
    const __nv_bfloat16* xr = x + t * ldx;
    for (int c = lane * 8; c < D; c += 256) {
      float xv[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr + c), xv);
#pragma unroll
      for (int e = 0; e < MAXE; ++e) {
        if (e < E) {
          float wv[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(router + (long long)e * D + c), wv);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[e] = fmaf(xv[j], wv[j], acc[e]);
        }
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      if (e < E) {
        acc[e] = warp_sum(acc[e]);   // every lane holds every logit
        mx = fmaxf(mx, acc[e]);
      }
    }
    float den = 0.f;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      if (e < E) {
        acc[e] = expf(acc[e] - mx);
        den += acc[e];
      }
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      if (e < E) {
        acc[e] *= inv;
        if ((e & 31) == lane) gates[t * E + e] = acc[e];
      }
    }
    // top-k by repeated arg-max; ties go to the lower expert index.  `best` starts at the lowest free
    // expert, so non-finite gates still yield k distinct, valid experts.
    unsigned long long taken = 0ull;
    for (int j = 0; j < k; ++j) {
      int best = __ffsll((long long)~taken) - 1;
      float bv = -1.f;
#pragma unroll
      for (int e = 0; e < MAXE; ++e) {
        if (e < E && !((taken >> e) & 1ull) && acc[e] > bv) {
          bv = acc[e];
          best = e;
        }
      }
      taken |= 1ull << best;
      if (lane == 0) topi[t * k + j] = best;
    }
  }
}

// ---------------------------------------------------------------- dispatch: one CTA of 1024 threads
// Stable counting sort of the M*k assignments (a = t*k + j, expert topi[a]) by expert: warp w walks
// the contiguous range [w*R, (w+1)*R) in 32-wide batches; within a batch __match_any_sync groups the
// lanes of one expert and a lane's rank is the number of lower lanes in its group.  Pass 1 counts per
// (warp, expert), a scan gives every (warp, expert) its first row, pass 2 writes the positions.  Also
// the balance-loss terms: coef[e] = E * frac_e and loss_acc += weight * sum_e mean_t(gate[t, e]) * coef[e].
template <int MAXE>
__global__ void __launch_bounds__(1024, 1)
    dispatch_kernel(const int* __restrict__ topi, const float* __restrict__ gates, int M, int k, int E, int cap,
                    int* __restrict__ seg, int* __restrict__ pos, int* __restrict__ src, float* __restrict__ rgate,
                    float* __restrict__ coef, float* __restrict__ loss_acc, float weight) {
  __shared__ int cnt[32][kMaxE + 1];   // per (warp, expert): count, then first row
  __shared__ int s_seg[kMaxE + 1];
  __shared__ float gsum[32][kMaxE + 1];
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int MK = M * k;
  const int R = (MK + 31) / 32;
  const int a0 = w * R, a1 = min(MK, a0 + R);
  const unsigned lt = (1u << lane) - 1u;
  for (int e = lane; e <= kMaxE; e += 32) cnt[w][e] = 0;
  __syncwarp();
  // the warp's expert ids, 8 batches of 32 at a time so that eight loads are in flight per lane
  // (clamped: a bad id cannot index out of range)
  auto load8 = [&](int b0, int (&ex)[8]) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int a = b0 + 32 * u + lane;
      ex[u] = a < a1 ? min(max(topi[a], 0), E - 1) : -1;
    }
  };
  // pass 1: counts
  for (int b0 = a0; b0 < a1; b0 += 256) {
    int exv[8];
    load8(b0, exv);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int ex = exv[u];
      const bool v = ex >= 0;
      const unsigned act = __ballot_sync(0xffffffffu, v);
      const unsigned peers = __match_any_sync(0xffffffffu, ex) & act;
      if (v && (peers & lt) == 0) cnt[w][ex] += __popc(peers);   // one leader per expert group
      __syncwarp();
    }
  }
  // gate sums for the balance loss (fixed order: per thread, then per warp, then over warps)
  {
    float acc[MAXE];
#pragma unroll
    for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
    for (int t = tid; t < M; t += 1024) {
#pragma unroll
      for (int e = 0; e < MAXE; ++e)
        if (e < E) acc[e] += gates[(long long)t * E + e];
    }
#pragma unroll
    for (int e = 0; e < MAXE; ++e) {
      if (e < E) {
        const float s = warp_sum(acc[e]);
        if (lane == 0) gsum[w][e] = s;
      }
    }
  }
  __syncthreads();
  // scan over warps per expert (thread (e, w') of a 32-lane row), then segment starts
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + w;   // warp w handles expert e, lane = source warp
    if (e < E) {
      int c = cnt[lane][e];
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      cnt[lane][e] = incl - c;                         // exclusive prefix within expert e
      if (lane == 31) s_seg[e + 1] = incl;             // total of expert e (temporarily)
    }
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    float bal = 0.f;
    for (int e = 0; e < E; ++e) {
      const int total = s_seg[e + 1];
      s_seg[e] = run;
      float gs = 0.f;
      for (int ww = 0; ww < 32; ++ww) gs += gsum[ww][e];
      const float c = (float)E * (float)total / (float)MK;
      coef[e] = c;
      bal += gs / (float)M * c;
      run += (total + kSeg - 1) / kSeg * kSeg;
      gsum[0][e] = (float)total;   // keep the count for the padding pass
    }
    s_seg[E] = run;
    if (loss_acc != nullptr) *loss_acc += weight * bal;
  }
  __syncthreads();
  for (int e = tid; e <= E; e += 1024) seg[e] = s_seg[e];
  // first row of every (warp, expert)
  for (int i = tid; i < 32 * E; i += 1024) {
    const int ww = i / E, e = i % E;
    cnt[ww][e] += s_seg[e];
  }
  __syncthreads();
  // pass 2: positions, source rows and gates of the sorted rows
  for (int b0 = a0; b0 < a1; b0 += 256) {
    int exv[8];
    load8(b0, exv);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int a = b0 + 32 * u + lane;
      const int ex = exv[u];
      const bool v = ex >= 0;
      const unsigned act = __ballot_sync(0xffffffffu, v);
      const unsigned peers = __match_any_sync(0xffffffffu, ex) & act;
      if (v) {
        const int p = cnt[w][ex] + __popc(peers & lt);
        const int t = a / k;
        pos[a] = p;
        src[p] = t;
        rgate[p] = gates[(long long)t * E + ex];
      }
      __syncwarp();
      if (v && (peers & lt) == 0) cnt[w][ex] += __popc(peers);
      __syncwarp();
    }
  }
  // padding rows of every segment and the rows past the last one
  for (int e = 0; e < E; ++e) {
    const int p0 = s_seg[e] + (int)gsum[0][e], p1 = s_seg[e + 1];
    for (int p = p0 + tid; p < p1; p += 1024) {
      src[p] = -1;
      rgate[p] = 0.f;
    }
  }
  for (int p = s_seg[E] + tid; p < cap; p += 1024) {
    src[p] = -1;
    rgate[p] = 0.f;
  }
}

// ---------------------------------------------------------------- gather: xs[p] = x[src[p]] (0 for padding)
__global__ void gather_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, const int* __restrict__ src,
                              const int* __restrict__ seg, int E, int D, __nv_bfloat16* __restrict__ xs) {
  const int used = seg[E];
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < used; p += warps) {
    const int t = src[p];
    uint4* dst = reinterpret_cast<uint4*>(xs + p * D);
    if (t >= 0) {
      const uint4* s = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
      for (int c = lane; c < D / 8; c += 32) dst[c] = s[c];
    } else {
      for (int c = lane; c < D / 8; c += 32) dst[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// ---------------------------------------------------------------- combine: out[t] = res[t] + sum_j gate_j ys[pos_j]
__global__ void combine_kernel(const float* __restrict__ res, const float* __restrict__ ys, const int* __restrict__ pos,
                               const float* __restrict__ rgate, int M, int k, int D, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < M; t += warps) {
    int p[kMaxK];
    float g[kMaxK];
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      if (j < k) {
        p[j] = pos[t * k + j];
        g[j] = rgate[p[j]];
      }
    }
    for (int c = lane * 4; c < D; c += 128) {
      float4 o = *reinterpret_cast<const float4*>(res + t * D + c);
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        if (j < k) {
          const float4 y = *reinterpret_cast<const float4*>(ys + (long long)p[j] * D + c);
          o.x = fmaf(g[j], y.x, o.x);
          o.y = fmaf(g[j], y.y, o.y);
          o.z = fmaf(g[j], y.z, o.z);
          o.w = fmaf(g[j], y.w, o.w);
        }
      }
      *reinterpret_cast<float4*>(out + t * D + c) = o;
    }
  }
}

// ---------------------------------------------------------------- combine backward, per sorted row:
// dys[p] = bf16(gate_p * dx[t]), dgate[p] = <dx[t], ys[p]> (0 and 0 for padding rows)
__global__ void combine_bwd_kernel(const float* __restrict__ dx, const float* __restrict__ ys, const int* __restrict__ src,
                                   const float* __restrict__ rgate, const int* __restrict__ seg, int E, int D,
                                   __nv_bfloat16* __restrict__ dys, float* __restrict__ dgate) {
  const int used = seg[E];
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < used; p += warps) {
    const int t = src[p];
    uint2* drow = reinterpret_cast<uint2*>(dys + p * D);
    if (t < 0) {
      for (int c = lane; c < D / 4; c += 32) drow[c] = make_uint2(0u, 0u);
      if (lane == 0) dgate[p] = 0.f;
      continue;
    }
    const float g = rgate[p];
    float dot = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      const float4 d = *reinterpret_cast<const float4*>(dx + (long long)t * D + c);
      const float4 y = *reinterpret_cast<const float4*>(ys + p * D + c);
      dot = fmaf(d.x, y.x, fmaf(d.y, y.y, fmaf(d.z, y.z, fmaf(d.w, y.w, dot))));
      drow[c >> 2] = make_uint2(pack_bf16x2(g * d.x, g * d.y), pack_bf16x2(g * d.z, g * d.w));
    }
    dot = warp_sum(dot);
    if (lane == 0) dgate[p] = dot;
  }
}

// ---------------------------------------------------------------- router backward, per token:
// dg[e] = weight * coef[e] / M + sum_j [topi_j == e] dgate[pos_j];  dlogit = gate * (dg - <gate, dg>);
// dn[t] = sum_j dxs[pos_j] + sum_e dlogit[e] router[e]
__global__ void router_bwd_kernel(const float* __restrict__ gates, const int* __restrict__ topi,
                                  const int* __restrict__ pos, const float* __restrict__ dgate,
                                  const float* __restrict__ coef, float weight, const float* __restrict__ dxs,
                                  const __nv_bfloat16* __restrict__ router, int M, int k, int E, int D,
                                  float* __restrict__ dlogits, float* __restrict__ dn) {
  __shared__ float s_dl[8][kMaxE];   // 8 warps per block
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long t = (long long)blockIdx.x * (blockDim.x >> 5) + wl; t < M; t += warps) {
    // lane holds experts lane and lane + 32
    float dg[2], gv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      dg[h] = e < E ? weight * coef[e] / (float)M : 0.f;
      gv[h] = e < E ? gates[t * E + e] : 0.f;
    }
    int p[kMaxK];
#pragma unroll
    for (int j = 0; j < kMaxK; ++j) {
      if (j < k) {
        p[j] = pos[t * k + j];
        const int e = topi[t * k + j];
        const float v = dgate[p[j]];
        if (e == lane) dg[0] += v;
        if (e == lane + 32) dg[1] += v;
      }
    }
    const float s = warp_sum(gv[0] * dg[0] + gv[1] * dg[1]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = lane + 32 * h;
      if (e < E) {
        const float dl = gv[h] * (dg[h] - s);
        dlogits[t * E + e] = dl;
        s_dl[wl][e] = dl;
      }
    }
    __syncwarp();
    for (int c = lane * 4; c < D; c += 128) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        if (j < k) {
          const float4 v = *reinterpret_cast<const float4*>(dxs + (long long)p[j] * D + c);
          o.x += v.x;
          o.y += v.y;
          o.z += v.z;
          o.w += v.w;
        }
      }
      for (int e = 0; e < E; ++e) {
        const float dl = s_dl[wl][e];
        const uint2 r = *reinterpret_cast<const uint2*>(router + (long long)e * D + c);
        o.x = fmaf(dl, bf16_lo(r.x), o.x);
        o.y = fmaf(dl, bf16_hi(r.x), o.y);
        o.z = fmaf(dl, bf16_lo(r.y), o.z);
        o.w = fmaf(dl, bf16_hi(r.y), o.w);
      }
      *reinterpret_cast<float4*>(dn + t * D + c) = o;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- router weight gradient:
// dR[e, d] += sum_t dlogits[t, e] x[t, d]; block = (128-token chunk, 256 columns), thread = column
template <int MAXE>
__global__ void router_wgrad_kernel(const float* __restrict__ dlogits, const __nv_bfloat16* __restrict__ x,
                                    long long ldx, int M, int E, int D, float* __restrict__ dR) {
  __shared__ float s_dl[128][MAXE];
  const int t0 = blockIdx.x * 128;
  const int d = blockIdx.y * 256 + threadIdx.x;
  const int nt = min(128, M - t0);
  for (int i = threadIdx.x; i < nt * E; i += 256) s_dl[i / E][i % E] = dlogits[(long long)(t0 + i / E) * E + i % E];
  __syncthreads();
  if (d >= D) return;
  float acc[MAXE];
#pragma unroll
  for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
  for (int i = 0; i < nt; ++i) {
    const float xv = __bfloat162float(x[(long long)(t0 + i) * ldx + d]);
#pragma unroll
    for (int e = 0; e < MAXE; ++e)
      if (e < E) acc[e] = fmaf(s_dl[i][e], xv, acc[e]);
  }
#pragma unroll
  for (int e = 0; e < MAXE; ++e)
    if (e < E) atomicAdd(dR + (long long)e * D + d, acc[e]);
}

// ---------------------------------------------------------------- per-expert column sums (bias gradients):
// db[e * N + n] += sum of rows of 256-row chunk c (every chunk lies in one expert's segment; padding
// rows are zero)
__global__ void seg_colsum_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ seg, int E, int N,
                                  float* __restrict__ db) {
  const int used = seg[E];
  const int r0 = blockIdx.x * kSeg;
  if (r0 >= used) return;
  int e = 0;
  while (e + 1 < E && seg[e + 1] <= r0) ++e;
  const int n = blockIdx.y * 256 + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int r = 0; r < kSeg; ++r) s += __bfloat162float(x[(long long)(r0 + r) * N + n]);
  atomicAdd(db + (long long)e * N + n, s);
}

}  // namespace moe
}  // namespace pcb

using namespace pcb;
using namespace pcb::moe;

static int grid_rows(long long rows, int warps_per_block) {
  long long b = (rows + warps_per_block - 1) / warps_per_block;
  return (int)(b < 148 * 16 ? (b < 1 ? 1 : b) : 148 * 16);
}

// the register arrays of the routing, dispatch and router-gradient kernels are sized for E rounded up
#define PCB_MOE_BY_E(E, CALL8, CALL16, CALL32, CALL64) \
  do {                                                 \
    if ((E) <= 8) CALL8;                               \
    else if ((E) <= 16) CALL16;                        \
    else if ((E) <= 32) CALL32;                        \
    else CALL64;                                       \
  } while (0)

int pcb_moe_route(const void* x, long long ldx, const void* router, int M, int D, int E, int k, float* gates,
                  int* topi, cudaStream_t s) {
  if (E < 1 || E > kMaxE || k < 1 || k > kMaxK || k > E || D % 8 != 0 || ldx % 8 != 0) return -1;
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* rb = reinterpret_cast<const __nv_bfloat16*>(router);
  const int grid = grid_rows(M, 8);
  PCB_MOE_BY_E(E, (route_kernel<8><<<grid, 256, 0, s>>>(xb, ldx, rb, M, D, E, k, gates, topi)),
               (route_kernel<16><<<grid, 256, 0, s>>>(xb, ldx, rb, M, D, E, k, gates, topi)),
               (route_kernel<32><<<grid, 256, 0, s>>>(xb, ldx, rb, M, D, E, k, gates, topi)),
               (route_kernel<64><<<grid, 256, 0, s>>>(xb, ldx, rb, M, D, E, k, gates, topi)));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_dispatch(const int* topi, const float* gates, int M, int k, int E, int cap, int* seg, int* pos, int* src,
                     float* rgate, float* coef, float* loss_acc, float weight, cudaStream_t s) {
  if (E < 1 || E > kMaxE || k < 1 || k > kMaxK) return -1;
  if ((long long)M * k + (long long)E * (kSeg - 1) > cap) return -1;
#define PCB_MOE_DISPATCH(X) \
  (dispatch_kernel<X><<<1, 1024, 0, s>>>(topi, gates, M, k, E, cap, seg, pos, src, rgate, coef, loss_acc, weight))
  PCB_MOE_BY_E(E, PCB_MOE_DISPATCH(8), PCB_MOE_DISPATCH(16), PCB_MOE_DISPATCH(32), PCB_MOE_DISPATCH(64));
#undef PCB_MOE_DISPATCH
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_gather(const void* x, long long ldx, const int* src, const int* seg, int E, int D, int cap, void* xs,
                   cudaStream_t s) {
  if (D % 8 != 0 || ldx % 8 != 0) return -1;
  gather_kernel<<<grid_rows(cap, 8), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, src, seg, E, D,
                                                  reinterpret_cast<__nv_bfloat16*>(xs));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_combine(const float* res, const float* ys, const int* pos, const float* rgate, int M, int k, int D,
                    float* out, cudaStream_t s) {
  if (D % 4 != 0 || k < 1 || k > kMaxK) return -1;
  combine_kernel<<<grid_rows(M, 8), 256, 0, s>>>(res, ys, pos, rgate, M, k, D, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_combine_bwd(const float* dx, const float* ys, const int* src, const float* rgate, const int* seg, int E,
                        int D, int cap, void* dys, float* dgate, cudaStream_t s) {
  if (D % 4 != 0) return -1;
  combine_bwd_kernel<<<grid_rows(cap, 8), 256, 0, s>>>(dx, ys, src, rgate, seg, E, D,
                                                       reinterpret_cast<__nv_bfloat16*>(dys), dgate);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_router_bwd(const float* gates, const int* topi, const int* pos, const float* dgate, const float* coef,
                       float weight, const float* dxs, const void* router, int M, int k, int E, int D, float* dlogits,
                       float* dn, cudaStream_t s) {
  if (E < 1 || E > kMaxE || k < 1 || k > kMaxK || D % 4 != 0) return -1;
  router_bwd_kernel<<<grid_rows(M, 8), 256, 0, s>>>(gates, topi, pos, dgate, coef, weight, dxs,
                                                    reinterpret_cast<const __nv_bfloat16*>(router), M, k, E, D,
                                                    dlogits, dn);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_router_wgrad(const float* dlogits, const void* x, long long ldx, int M, int E, int D, float* dR,
                         cudaStream_t s) {
  if (E < 1 || E > kMaxE) return -1;
  const dim3 grid((M + 127) / 128, (D + 255) / 256);
  const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
#define PCB_MOE_RW(X) (router_wgrad_kernel<X><<<grid, 256, 0, s>>>(dlogits, xb, ldx, M, E, D, dR))
  PCB_MOE_BY_E(E, PCB_MOE_RW(8), PCB_MOE_RW(16), PCB_MOE_RW(32), PCB_MOE_RW(64));
#undef PCB_MOE_RW
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_moe_seg_colsum(const void* x, const int* seg, int E, int N, int cap, float* db, cudaStream_t s) {
  const dim3 grid((cap + kSeg - 1) / kSeg, (N + 255) / 256);
  seg_colsum_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), seg, E, N, db);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
