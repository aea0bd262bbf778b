// Serving and small-op kernels: split-KV decode attention, weight-only int8/int4 GEMV,
// row softmax forward/backward and the gated linear recurrence scan.
//
// Reference counterparts: PredictiveCoding.Device/Kernels/DeviceMath.cs:134-158 (attn_1q: one
// thread per head, whole cache serially), :58-71 / :218-226 (softmax rows with one thread per
// row), PredictiveCoding.LLM/Infrastructure/Quantization.cs:1-135 (Int8/Int4 matvec on the host)
// and Autograd.cs:741-767 (RecurrentScan on the host).
//
// decode attention: flash-decoding.  One CTA per (split, kv-head, sequence) walks a contiguous
// slice of the cache for all G query heads that share that kv head (GQA), keeps an online-softmax
// state per warp, merges its 4 warps in shared memory and writes (m, l, acc) for the split; a
// second launch merges the splits (with one split the CTA writes the output itself).  Keys are scored lane-per-key (no shuffles in the dot product),
// values are accumulated lane-per-dimension (coalesced 2*HD-byte rows) and requested early (half of a
// tile's value rows together with its keys, the other half right after the key math), so K and V are
// each read once from HBM in little more than one memory round trip per tile.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>

#include "common.cuh"

using namespace pcb;

namespace {

constexpr int kDecWarps = 4;

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

template <int HD, int G>
__global__ void __launch_bounds__(kDecWarps * 32)
decode_attn_split_kernel(const __nv_bfloat16* __restrict__ q,      // [B, H, HD]
                         const __nv_bfloat16* __restrict__ kc,     // [B, Hkv, cap, HD]
                         const __nv_bfloat16* __restrict__ vc,     // [B, Hkv, cap, HD]
                         const int* __restrict__ lens,             // [B]
                         float* __restrict__ part_acc,             // [B, H, nsplit, HD]
                         float* __restrict__ part_ml,              // [B, H, nsplit, 2]
                         __nv_bfloat16* __restrict__ out,          // [B, H, HD], written when nsplit == 1
                         int Hkv, int cap, int nsplit, float scale, float softcap) {
  pdl_begin();
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int H = Hkv * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = lens[b];
  const int per = (len + nsplit - 1) / nsplit;
  const int t0 = split * per, t1 = min(len, t0 + per);

  __shared__ float sq[G][HD];
  __shared__ float sm_m[kDecWarps][G], sm_l[kDecWarps][G];
  __shared__ float sacc[kDecWarps][G][HD];
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    int hh = i / HD, d = i % HD;
    sq[hh][d] = bf(q[((long long)b * H + g * G + hh) * HD + d]) * scale;
  }
  __syncthreads();

  const long long kvbase = ((long long)b * Hkv + g) * cap * HD;
  constexpr int DPL = HD / 32;                      // dims per lane in the V phase
  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[hh][j] = 0.f;
  }

  __shared__ float ssc[kDecWarps][G][32];
  constexpr int LPK = HD / 8;                     // lanes per key row (16 for HD 128, 8 for HD 64)
  constexpr int KPS = 32 / LPK;                   // keys per warp step
  constexpr int STEPS = 32 / KPS;
  const int sub = lane / LPK, c = lane % LPK;
  // this lane's 8 query dims (c * 8 ..) stay in registers for one or two heads
  constexpr bool QREG = G <= 2;
  float qr[QREG ? G : 1][8];
  if constexpr (QREG) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh)
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[hh][e] = sq[hh][c * 8 + e];
  }
  using VRaw = typename std::conditional<DPL == 4, uint2, uint32_t>::type;
  for (int tile = t0 + warp * 32; tile < t1; tile += kDecWarps * 32) {
    // scores: half-warps take one key row each (HD/8 lanes x 16 bytes, coalesced), two rows per step;
    // the partial dot products are reduced across the half-warp and parked in shared memory.  The first
    // 16 value rows are requested together with the keys and the other 16 right after the key math, so a
    // tile costs little more than one memory round trip; rows past the slice repeat its last row
    // (weight 0).
    const int nk = min(32, t1 - tile);
    uint4 raw_all[STEPS];
#pragma unroll
    for (int it = 0; it < STEPS; ++it) {
      const int t = tile + it * KPS + sub;
      raw_all[it] = t < t1 ? __ldg(reinterpret_cast<const uint4*>(kc + kvbase + (long long)t * HD) + c)
                           : make_uint4(0u, 0u, 0u, 0u);
    }
    // (with four or eight heads per kv head the registers go to the per-head state: values follow the
    // softmax in batches of eight rows instead)
    constexpr bool EARLY_V = G <= 2;
    VRaw va[EARLY_V ? 16 : 1], vb[EARLY_V ? 16 : 1];
    if constexpr (EARLY_V) {
#pragma unroll
      for (int u = 0; u < 16; ++u)
        va[u] = __ldg(reinterpret_cast<const VRaw*>(vc + kvbase + (long long)(tile + min(u, nk - 1)) * HD +
                                                    lane * DPL));
    }
#pragma unroll
    for (int it = 0; it < STEPS; ++it) {
      const int kk = it * KPS;
      float part[G];
#pragma unroll
      for (int hh = 0; hh < G; ++hh) part[hh] = 0.f;
      {
        const uint4 raw = raw_all[it];
        const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kv = __bfloat1622float2(p2[e]);
#pragma unroll
          for (int hh = 0; hh < G; ++hh) {
            if constexpr (QREG) part[hh] += qr[hh][2 * e] * kv.x + qr[hh][2 * e + 1] * kv.y;
            else part[hh] += sq[hh][c * 8 + 2 * e] * kv.x + sq[hh][c * 8 + 2 * e + 1] * kv.y;
          }
        }
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], o);
        if (c == 0) ssc[warp][hh][kk + sub] = part[hh];
      }
    }
    if constexpr (EARLY_V) {
#pragma unroll
      for (int u = 0; u < 16; ++u)
        vb[u] = __ldg(reinterpret_cast<const VRaw*>(vc + kvbase + (long long)(tile + min(16 + u, nk - 1)) * HD +
                                                    lane * DPL));
    }
    __syncwarp();
    const int t = tile + lane;
    float s[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      s[hh] = t < t1 ? ssc[warp][hh][lane] : -INFINITY;
      if (t < t1 && softcap > 0.f) s[hh] = softcap * tanhf(s[hh] / softcap);
    }
    __syncwarp();
    // online softmax over this 32-key tile, per head
    float p[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float tmax = warp_max(s[hh]);
      float mnew = fmaxf(m[hh], tmax);
      float corr = (m[hh] == -INFINITY) ? 0.f : __expf(m[hh] - mnew);
      p[hh] = (s[hh] == -INFINITY) ? 0.f : __expf(s[hh] - mnew);
      l[hh] = l[hh] * corr + warp_sum(p[hh]);
      m[hh] = mnew;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[hh][j] *= corr;
    }
    auto pv = [&](const VRaw& raw, int u) {
      float vv[DPL];
      if constexpr (DPL == 4) {
        const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        vv[0] = a0.x; vv[1] = a0.y; vv[2] = a1.x; vv[3] = a1.y;
      } else {
        const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw));
        vv[0] = a0.x; vv[1] = a0.y;
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        const float pk = __shfl_sync(0xffffffffu, p[hh], u);   // 0 for keys past the slice
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[hh][j] += pk * vv[j];
      }
    };
    if constexpr (EARLY_V) {
#pragma unroll
      for (int u = 0; u < 16; ++u) pv(va[u], u);
#pragma unroll
      for (int u = 0; u < 16; ++u) pv(vb[u], 16 + u);
    } else {
      for (int k0 = 0; k0 < nk; k0 += 8) {       // eight value rows in flight at a time
        VRaw vr[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          vr[u] = __ldg(reinterpret_cast<const VRaw*>(vc + kvbase + (long long)(tile + min(k0 + u, nk - 1)) * HD +
                                                      lane * DPL));
#pragma unroll
        for (int u = 0; u < 8; ++u) pv(vr[u], k0 + u);
      }
    }
  }
  // merge the warps
  if (lane == 0) {
#pragma unroll
    for (int hh = 0; hh < G; ++hh) { sm_m[warp][hh] = m[hh]; sm_l[warp][hh] = l[hh]; }
  }
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
#pragma unroll
    for (int j = 0; j < DPL; ++j) sacc[warp][hh][lane * DPL + j] = acc[hh][j];
  __syncthreads();
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
    const int hh = i / HD, d = i % HD;
    float mm = -INFINITY;
    for (int w = 0; w < kDecWarps; ++w) mm = fmaxf(mm, sm_m[w][hh]);
    float ll = 0.f, a = 0.f;
    for (int w = 0; w < kDecWarps; ++w) {
      float c = (sm_m[w][hh] == -INFINITY) ? 0.f : __expf(sm_m[w][hh] - mm);
      ll += sm_l[w][hh] * c;
      a += sacc[w][hh][d] * c;
    }
    if (nsplit == 1) {
      // one split: this CTA has the whole row, so it writes the output (no merge launch)
      out[((long long)b * H + g * G + hh) * HD + d] = __float2bfloat16(ll > 0.f ? a / ll : 0.f);
    } else {
      const long long row = ((long long)b * H + g * G + hh) * nsplit + split;
      part_acc[row * HD + d] = a;
      if (d == 0) { part_ml[row * 2] = mm; part_ml[row * 2 + 1] = ll; }
    }
  }
}

template <int HD>
__global__ void decode_attn_combine_kernel(const float* __restrict__ part_acc, const float* __restrict__ part_ml,
                                           __nv_bfloat16* __restrict__ out, int nsplit) {
  pdl_begin();
  const long long bh = blockIdx.x;                 // b * H + h
  const int d = threadIdx.x;
  float mm = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mm = fmaxf(mm, part_ml[(bh * nsplit + s) * 2]);
  float ll = 0.f, a = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    float ms = part_ml[(bh * nsplit + s) * 2];
    float c = (ms == -INFINITY) ? 0.f : __expf(ms - mm);
    ll += part_ml[(bh * nsplit + s) * 2 + 1] * c;
    if (d < HD) a += part_acc[(bh * nsplit + s) * HD + d] * c;
  }
  if (d < HD) out[bh * HD + d] = __float2bfloat16(ll > 0.f ? a / ll : 0.f);
}

// ------------------------------------------------------------------ weight-only GEMV
// y[b, r] = scale[r] * sum_c x[b, c] * q[r, c] for NB <= 8 activation rows.  One warp owns
// kRows rows; each lane loads 8 bytes of every row per step (8 int8 or 16 int4 weights), the
// activations for those columns are loaded once and reused across the kRows rows.
constexpr int kGemvRows = 4;

template <int BITS, int NB>
__global__ void __launch_bounds__(256)
wq_gemv_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w, const float* __restrict__ scale,
               float* __restrict__ y, int rows, int cols) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int r0 = warp * kGemvRows;
  if (r0 >= rows) return;
  constexpr int VPL = BITS == 8 ? 8 : 16;          // weights per 8-byte load
  const long long row_bytes = BITS == 8 ? cols : cols / 2;
  float acc[kGemvRows][NB];
#pragma unroll
  for (int i = 0; i < kGemvRows; ++i)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[i][b] = 0.f;
  for (int c0 = lane * VPL; c0 < cols; c0 += 32 * VPL) {
    uint2 wr[kGemvRows];
#pragma unroll
    for (int i = 0; i < kGemvRows; ++i) {
      const int r = min(r0 + i, rows - 1);
      wr[i] = __ldg(reinterpret_cast<const uint2*>(w + r * row_bytes + (BITS == 8 ? c0 : c0 / 2)));
    }
#pragma unroll
    for (int half = 0; half < VPL / 8; ++half) {
      float xv[NB][8];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float4* xp = reinterpret_cast<const float4*>(x + (long long)b * cols + c0 + half * 8);
        float4 u = __ldg(xp), v = __ldg(xp + 1);
        xv[b][0] = u.x; xv[b][1] = u.y; xv[b][2] = u.z; xv[b][3] = u.w;
        xv[b][4] = v.x; xv[b][5] = v.y; xv[b][6] = v.z; xv[b][7] = v.w;
      }
#pragma unroll
      for (int i = 0; i < kGemvRows; ++i) {
        float wf[8];
        if constexpr (BITS == 8) {
          const int8_t* q8 = reinterpret_cast<const int8_t*>(&wr[i]);
#pragma unroll
          for (int e = 0; e < 8; ++e) wf[e] = static_cast<float>(q8[e]);
        } else {
          const uint32_t word = half == 0 ? wr[i].x : wr[i].y;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            int nib = (word >> (4 * e)) & 0xF;
            wf[e] = static_cast<float>(nib >= 8 ? nib - 16 : nib);
          }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[i][b] += wf[e] * xv[b][e];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kGemvRows; ++i) {
    const int r = r0 + i;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float s = warp_sum(acc[i][b]);
      if (lane == 0 && r < rows) y[(long long)b * rows + r] = s * scale[r];
    }
  }
}

// ------------------------------------------------------------------ row softmax
// One warp per row for rows up to 32*32 elements held in registers; longer rows use a
// three-pass loop (max, sum, write).  y = softmax(x * scale) with -inf entries mapping to 0.
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, int n, float scale) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (long long)row * n;
  float* yr = y + (long long)row * n;
  float mx = -INFINITY;
  for (int i = lane; i < n; i += 32) mx = fmaxf(mx, xr[i] * scale);
  mx = warp_max(mx);
  float s = 0.f;
  for (int i = lane; i < n; i += 32) s += (mx == -INFINITY) ? 0.f : __expf(xr[i] * scale - mx);
  s = warp_sum(s);
  const float inv = s > 0.f ? 1.f / s : 0.f;
  for (int i = lane; i < n; i += 32) yr[i] = (mx == -INFINITY) ? 0.f : __expf(xr[i] * scale - mx) * inv;
}

// dx = y * (dy - sum(dy * y)) * scale
__global__ void softmax_rows_bwd_kernel(const float* __restrict__ y, const float* __restrict__ dy,
                                        float* __restrict__ dx, int rows, int n, float scale) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long o = (long long)row * n;
  float dot = 0.f;
  for (int i = lane; i < n; i += 32) dot += dy[o + i] * y[o + i];
  dot = warp_sum(dot);
  for (int i = lane; i < n; i += 32) dx[o + i] = y[o + i] * (dy[o + i] - dot) * scale;
}

// ------------------------------------------------------------------ gated linear recurrence
// s_t = a_t * s_{t-1} + b_t over t for every (batch, channel); [B, T, D] row-major.  One thread
// per channel walks T: every element is read once and consecutive threads read consecutive
// channels, so the scan runs at HBM speed without a parallel-prefix formulation.
__global__ void linear_scan_fwd_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                       float* __restrict__ s, int B, int T, int D) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)B * D) return;
  const int bb = idx / D, d = idx % D;
  const long long base = (long long)bb * T * D + d;
  float st = 0.f;
  for (int t = 0; t < T; ++t) {
    const long long o = base + (long long)t * D;
    st = a[o] * st + b[o];
    s[o] = st;
  }
}

// g_t = ds_t + a_{t+1} g_{t+1};  da_t = g_t * s_{t-1};  db_t = g_t
__global__ void linear_scan_bwd_kernel(const float* __restrict__ a, const float* __restrict__ s,
                                       const float* __restrict__ ds, float* __restrict__ da, float* __restrict__ db,
                                       int B, int T, int D) {
  const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (idx >= (long long)B * D) return;
  const int bb = idx / D, d = idx % D;
  const long long base = (long long)bb * T * D + d;
  float g = 0.f;
  for (int t = T - 1; t >= 0; --t) {
    const long long o = base + (long long)t * D;
    g = ds[o] + (t + 1 < T ? a[o + D] * g : 0.f);
    db[o] = g;
    da[o] = t > 0 ? g * s[o - D] : 0.f;
  }
}

template <int HD>
int launch_decode(const __nv_bfloat16* q, const __nv_bfloat16* kc, const __nv_bfloat16* vc, const int* lens,
                  float* pacc, float* pml, __nv_bfloat16* out, int B, int Hkv, int G, int cap, int nsplit,
                  float scale, float softcap, cudaStream_t s) {
  dim3 grid(nsplit, Hkv, B);
  switch (G) {
#define PCB_DEC_CASE(GG)                                                                                       \
  case GG:                                                                                                     \
    pdl_launch(decode_attn_split_kernel<HD, GG>, grid, dim3(kDecWarps * 32), 0, s, q, kc, vc, lens, pacc, pml, \
               out, Hkv, cap, nsplit, scale, softcap);                                                         \
    break;
    PCB_DEC_CASE(1) PCB_DEC_CASE(2) PCB_DEC_CASE(4) PCB_DEC_CASE(8)
#undef PCB_DEC_CASE
    default: return -2;
  }
  if (nsplit > 1)
    pdl_launch(decode_attn_combine_kernel<HD>, dim3(B * Hkv * G), dim3(HD), 0, s, pacc, pml, out, nsplit);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// One decode token per row: rotate q and k of qkv [B, 3*H*HD] (RoPE angle table row cs [HD/2]
// float2 for position *pos), write q to qo [B, H, HD] and append k, v to the caches at *pos.
__global__ void rope_append_kernel(const __nv_bfloat16* __restrict__ qkv, const float2* __restrict__ cs_table,
                                   const long long* __restrict__ pos, __nv_bfloat16* __restrict__ qo,
                                   __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int H, int HD,
                                   int cap) {
  pdl_begin();
  const int b = blockIdx.x;
  const long long p = *pos;
  const int D = H * HD;
  const __nv_bfloat16* row = qkv + (long long)b * 3 * D;
  const float2* cs = cs_table + p * (HD / 2);
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {  // pair i of q and of k
    const int h = (2 * i) / HD, d = (2 * i) % HD;
    const float2 c = cs[d / 2];
    const float2 qv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row)[i]);
    const float2 kv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row + D)[i]);
    reinterpret_cast<__nv_bfloat162*>(qo + (long long)b * D)[i] =
        __floats2bfloat162_rn(qv.x * c.x - qv.y * c.y, qv.x * c.y + qv.y * c.x);
    const long long o = (((long long)b * H + h) * cap + p) * HD + d;
    *reinterpret_cast<__nv_bfloat162*>(kc + o) = __floats2bfloat162_rn(kv.x * c.x - kv.y * c.y, kv.x * c.y + kv.y * c.x);
    *reinterpret_cast<__nv_bfloat162*>(vc + o) = reinterpret_cast<const __nv_bfloat162*>(row + 2 * D)[i];
  }
}

// a[r, j] = silu(gu[r, j]) * gu[r, F + j] for gu [rows, 2F] bf16 (gate | up), a [rows, F] bf16
__global__ void swiglu_rows_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a, int rows,
                                   int F, int il16) {
  pdl_begin();
  const long long n = (long long)rows * F;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / F;
    const int j = (int)(i % F);
    // gate | up halves, or alternating blocks of 16 gate and 16 up columns
    const long long gi = r * 2 * F + (il16 ? (j >> 4) * 32 + (j & 15) : j);
    const float g = __bfloat162float(gu[gi]);
    const float u = __bfloat162float(gu[gi + (il16 ? 16 : F)]);
    a[i] = __float2bfloat16(g / (1.f + __expf(-g)) * u);
  }
}

}  // namespace

// q [B, H, HD] bf16; caches [B, Hkv, cap, HD] bf16; lens [B] int32 (valid entries);
// scratch pacc [B, H, nsplit, HD] fp32 and pml [B, H, nsplit, 2] fp32; out [B, H, HD] bf16.
int pcb_decode_attn(const void* q, const void* kc, const void* vc, const int* lens, float* pacc, float* pml,
                    void* out, int B, int H, int Hkv, int HD, int cap, int nsplit, float scale, float softcap,
                    cudaStream_t s) {
  if (Hkv <= 0 || H % Hkv) return -2;
  const int G = H / Hkv;
  auto q16 = reinterpret_cast<const __nv_bfloat16*>(q);
  auto k16 = reinterpret_cast<const __nv_bfloat16*>(kc);
  auto v16 = reinterpret_cast<const __nv_bfloat16*>(vc);
  auto o16 = reinterpret_cast<__nv_bfloat16*>(out);
  if (HD == 64) return launch_decode<64>(q16, k16, v16, lens, pacc, pml, o16, B, Hkv, G, cap, nsplit, scale, softcap, s);
  if (HD == 128) return launch_decode<128>(q16, k16, v16, lens, pacc, pml, o16, B, Hkv, G, cap, nsplit, scale, softcap, s);
  return -2;
}

// x [NB, cols] fp32; w [rows, cols] int8 or [rows, cols/2] packed int4; scale [rows]; y [NB, rows].
int pcb_wq_gemv(const float* x, const void* w, const float* scale, float* y, int NB, int rows, int cols, int bits,
                cudaStream_t s) {
  if (cols % (bits == 8 ? 8 : 16) || NB < 1 || NB > 8) return -2;
  const int warps = (rows + kGemvRows - 1) / kGemvRows;
  const int grid = (warps * 32 + 255) / 256;
  auto w8 = reinterpret_cast<const uint8_t*>(w);
#define PCB_GEMV(BITS, NBV) wq_gemv_kernel<BITS, NBV><<<grid, 256, 0, s>>>(x, w8, scale, y, rows, cols)
#define PCB_GEMV_NB(BITS)                                                  \
  switch (NB) {                                                            \
    case 1: PCB_GEMV(BITS, 1); break;                                      \
    case 2: PCB_GEMV(BITS, 2); break;                                      \
    case 3: PCB_GEMV(BITS, 3); break;                                      \
    case 4: PCB_GEMV(BITS, 4); break;                                      \
    case 5: PCB_GEMV(BITS, 5); break;                                      \
    case 6: PCB_GEMV(BITS, 6); break;                                      \
    case 7: PCB_GEMV(BITS, 7); break;                                      \
    default: PCB_GEMV(BITS, 8); break;                                     \
  }
  if (bits == 8) { PCB_GEMV_NB(8) } else { PCB_GEMV_NB(4) }
#undef PCB_GEMV_NB
#undef PCB_GEMV
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_softmax_rows(const float* x, float* y, int rows, int n, float scale, cudaStream_t s) {
  softmax_rows_kernel<<<(rows * 32 + 255) / 256, 256, 0, s>>>(x, y, rows, n, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_softmax_rows_bwd(const float* y, const float* dy, float* dx, int rows, int n, float scale, cudaStream_t s) {
  softmax_rows_bwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, s>>>(y, dy, dx, rows, n, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_linear_scan(const float* a, const float* b, float* st, int B, int T, int D, cudaStream_t s) {
  const long long n = (long long)B * D;
  linear_scan_fwd_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, b, st, B, T, D);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_linear_scan_bwd(const float* a, const float* st, const float* ds, float* da, float* db, int B, int T, int D,
                        cudaStream_t s) {
  const long long n = (long long)B * D;
  linear_scan_bwd_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, st, ds, da, db, B, T, D);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_rope_append(const void* qkv, const float* cs_table, const long long* pos, void* qo, void* kc, void* vc, int B,
                    int H, int HD, int cap, cudaStream_t s) {
  if (HD % 2 || B <= 0) return -2;
  pdl_launch(rope_append_kernel, dim3(B), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(qkv),
             reinterpret_cast<const float2*>(cs_table), pos, reinterpret_cast<__nv_bfloat16*>(qo),
             reinterpret_cast<__nv_bfloat16*>(kc), reinterpret_cast<__nv_bfloat16*>(vc), H, HD, cap);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_swiglu_rows(const void* gu, void* a, int rows, int F, int il16, cudaStream_t s) {
  if (il16 && F % 16) return -2;
  const long long n = (long long)rows * F;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  pdl_launch(swiglu_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(gu),
             reinterpret_cast<__nv_bfloat16*>(a), rows, F, il16);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
