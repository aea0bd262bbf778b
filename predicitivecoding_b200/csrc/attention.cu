// Causal flash attention forward / backward for the fused decoder trainer.
//
// Replaces the reference's attn_fwd / attn_dot / attn_bwd_dq / attn_bwd_dkv
// (PredictiveCoding.Device/Kernels/DeviceTrainKernels.cs:272-480), which run one block
// per (query, head) in fp32 SIMT and never reuse K/V across queries.  Here one CTA
// owns a tile of queries (forward) or keys (backward) and streams the other side
// through double-buffered shared memory with cp.async; products run on the tensor
// cores (bf16 in, fp32 accumulate); the softmax is the online (running max / sum)
// form and the backward replays P from the saved log-sum-exp, as the reference does.
//
// Layout: q, k, v live in one fused activation buffer [B*S, ld] (bf16) at column
// offsets 0, D, 2D, head h at h*hd; the output is [B*S, ld_o].  lse is [B*H, S].
#include <cstdint>

#include "common.cuh"

namespace pcb {
namespace attn {

PCB_DEVICE void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
PCB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
PCB_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

PCB_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
PCB_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
PCB_DEVICE void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Swizzled [rows][HD] bf16 tile: 16-byte chunk c of row r lives at chunk (c ^ (r & 7)).
template <int HD>
PCB_DEVICE uint32_t tile_off(int r, int c) {
  return static_cast<uint32_t>(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

// Copy a [ROWS][HD] tile from global rows (stride ld elements) into swizzled smem.
template <int HD, int ROWS, int NT>
PCB_DEVICE void load_tile(uint32_t sbase, const __nv_bfloat16* g, long long ld, int tid) {
  constexpr int CH = HD / 8;
#pragma unroll
  for (int i = tid; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    cp_async16(sbase + tile_off<HD>(r, c), g + r * ld + c * 8);
  }
}

// ------------------------------------------------------------------------------------------
// forward:  one CTA = BQ = 16*NW queries of one (batch, head); KV blocks of 64.
// ------------------------------------------------------------------------------------------
template <int HD, int NW>
__global__ void __launch_bounds__(NW * 32)
    attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, long long ld, __nv_bfloat16* __restrict__ out,
                    long long ld_o, float* __restrict__ lse, int S, int H, float scale) {
  constexpr int BQ = 16 * NW, BKV = 64, NT = NW * 32;
  constexpr int KSTEPS = HD / 16;  // k-steps over head dim
  constexpr int DT = HD / 8;       // output n-tiles
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BQ * HD * 2;
  const uint32_t sV0 = sK0 + 2 * BKV * HD * 2;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  // heavy (late) query tiles first: better tail balance under the causal mask
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int D = H * HD;
  const long long row0 = (long long)b * S;
  const int q0 = qb * BQ;
  const __nv_bfloat16* Qg = qkv + (row0 + q0) * ld + h * HD;
  const __nv_bfloat16* Kg = qkv + row0 * ld + D + h * HD;
  const __nv_bfloat16* Vg = qkv + row0 * ld + 2 * D + h * HD;

  const int kv_end = min(S, q0 + BQ);
  const int nkv = (kv_end + BKV - 1) / BKV;

  load_tile<HD, BQ, NT>(sQ, Qg, ld, tid);
  load_tile<HD, BKV, NT>(sK0, Kg, ld, tid);
  load_tile<HD, BKV, NT>(sV0, Vg, ld, tid);
  cp_async_commit();

  uint32_t qf[KSTEPS][4];
  float o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = scale * 1.4426950408889634f;

  for (int j = 0; j < nkv; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkv) {
      load_tile<HD, BKV, NT>(sK0 + (buf ^ 1) * BKV * HD * 2, Kg + (long long)(j + 1) * BKV * ld, ld, tid);
      load_tile<HD, BKV, NT>(sV0 + (buf ^ 1) * BKV * HD * 2, Vg + (long long)(j + 1) * BKV * ld, ld, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sQ + tile_off<HD>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint32_t sK = sK0 + buf * BKV * HD * 2;
    const uint32_t sV = sV0 + buf * BKV * HD * 2;
    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
        const int idx = lane >> 3;
        const int r = np * 16 + (idx >> 1) * 8 + (lane & 7);
        const int c = kk * 2 + (idx & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // causal mask (only the diagonal block needs it)
    const int kbase = j * BKV;
    const int qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;
    if (kbase + BKV > q0) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int kc = kbase + nt * 8 + 2 * t;
        if (kc > qr0) s[nt][0] = -INFINITY;
        if (kc + 1 > qr0) s[nt][1] = -INFINITY;
        if (kc > qr1) s[nt][2] = -INFINITY;
        if (kc + 1 > qr1) s[nt][3] = -INFINITY;
      }
    }
    // online softmax
    float mx0 = mrow[0], mx1 = mrow[1];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = (mrow[0] == -INFINITY) ? 0.f : exp2f((mrow[0] - mx0) * sl2);
    const float c1 = (mrow[1] == -INFINITY) ? 0.f : exp2f((mrow[1] - mx1) * sl2);
    mrow[0] = mx0;
    mrow[1] = mx1;
    const float ms0 = mx0 * sl2, ms1 = mx1 * sl2;
    float ls0 = 0.f, ls1 = 0.f;
    uint32_t pf[4][4];  // P as A fragments (4 k-steps of 16 keys)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] * sl2 - ms0);
      const float p1 = exp2f(s[nt][1] * sl2 - ms0);
      const float p2 = exp2f(s[nt][2] * sl2 - ms1);
      const float p3 = exp2f(s[nt][3] * sl2 - ms1);
      ls0 += p0 + p1;
      ls1 += p2 + p3;
      const int kk = nt >> 1, hi = nt & 1;
      pf[kk][hi * 2 + 0] = pack_bf16x2(p0, p1);
      pf[kk][hi * 2 + 1] = pack_bf16x2(p2, p3);
    }
    lrow[0] = lrow[0] * c0 + ls0;
    lrow[1] = lrow[1] * c1 + ls1;
#pragma unroll
    for (int dt = 0; dt < DT; ++dt) {
      o[dt][0] *= c0; o[dt][1] *= c0;
      o[dt][2] *= c1; o[dt][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int idx = lane >> 3;
        const int r = kk * 16 + (idx & 1) * 8 + (lane & 7);
        const int c = dp * 2 + (idx >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(o[2 * dp], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b0, b1);
        mma16816(o[2 * dp + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b2, b3);
      }
    }
    __syncthreads();
  }
  // finalize
  float l0 = lrow[0], l1 = lrow[1];
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int qr0 = q0 + warp * 16 + g;
  __nv_bfloat16* o0 = out + (row0 + qr0) * ld_o + h * HD;
  __nv_bfloat16* o1 = o0 + 8 * ld_o;
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int c = dt * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(o0 + c) = pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
    *reinterpret_cast<uint32_t*>(o1 + c) = pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
  if (t == 0) {
    lse[(long long)bh * S + qr0] = mrow[0] * scale + logf(l0);
    lse[(long long)bh * S + qr0 + 8] = mrow[1] * scale + logf(l1);
  }
}

// ------------------------------------------------------------------------------------------
// backward preprocess: Dv[bh, i] = sum_d dO[i,d] * O[i,d];  zero the fp32 dQ accumulator.
// ------------------------------------------------------------------------------------------
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                    long long ld_o, float* __restrict__ dvec, float* __restrict__ dq_acc, int B,
                                    int S, int H, int HD) {
  const int warps = blockDim.x >> 5;
  const long long idx = (long long)blockIdx.x * warps + (threadIdx.x >> 5);  // (b*S + i)*H + h
  const int lane = threadIdx.x & 31;
  if (idx >= (long long)B * S * H) return;
  const int h = (int)(idx % H);
  const long long row = idx / H;
  const int b = (int)(row / S), i = (int)(row % S);
  const __nv_bfloat16* op = o + row * ld_o + h * HD;
  const __nv_bfloat16* dp = dout + row * ld_o + h * HD;
  float s = 0.f;
  for (int d = lane * 2; d < HD; d += 64) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(op + d));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dp + d));
    s += a.x * c.x + a.y * c.y;
  }
  s = warp_sum(s);
  if (lane == 0) dvec[((long long)b * H + h) * S + i] = s;
  float* dq = dq_acc + row * (long long)(H * HD) + h * HD;
  for (int d = lane; d < HD; d += 32) dq[d] = 0.f;
}

// ------------------------------------------------------------------------------------------
// backward main: one CTA = 64 keys (4 warps x 16 keys) of one (batch, head); query blocks of BQ.
// dK, dV stay in registers; dQ partials go to an fp32 accumulator with atomics.
// ------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(128)
    attn_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, long long ld, const __nv_bfloat16* __restrict__ dout,
                    long long ld_o, const float* __restrict__ lse, const float* __restrict__ dvec,
                    float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long long ld_d, int S, int H,
                    float scale, const float2* __restrict__ rope_cs) {
  constexpr int BKV = 64, BQ = 64, NT = 128;
  constexpr int KSTEPS = HD / 16;
  constexpr int DT = HD / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BKV * HD * 2;
  const uint32_t sQ0 = sV + BKV * HD * 2;           // 2 buffers
  const uint32_t sO0 = sQ0 + 2 * BQ * HD * 2;       // 2 buffers (dO)
  const uint32_t sdS = sO0 + 2 * BQ * HD * 2;       // [BQ][BKV] bf16, swizzled as HD=64 tile
  float* sL = reinterpret_cast<float*>(smem + (sdS - sK) + BQ * BKV * 2);  // 2 x BQ
  float* sDv = sL + 2 * BQ;                                                // 2 x BQ

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int D = H * HD;
  const long long row0 = (long long)b * S;
  const int k0 = kb * BKV;

  const __nv_bfloat16* Kg = qkv + (row0 + k0) * ld + D + h * HD;
  const __nv_bfloat16* Vg = qkv + (row0 + k0) * ld + 2 * D + h * HD;
  const __nv_bfloat16* Qg = qkv + row0 * ld + h * HD;
  const __nv_bfloat16* dOg = dout + row0 * ld_o + h * HD;
  const float* Lg = lse + (long long)bh * S;
  const float* Dg = dvec + (long long)bh * S;

  const int qb_begin = k0 / BQ;
  const int nqb = (S + BQ - 1) / BQ;
  const float sl2 = scale * 1.4426950408889634f;

  load_tile<HD, BKV, NT>(sK, Kg, ld, tid);
  load_tile<HD, BKV, NT>(sV, Vg, ld, tid);
  auto load_q = [&](int qb, int buf) {
    load_tile<HD, BQ, NT>(sQ0 + buf * BQ * HD * 2, Qg + (long long)qb * BQ * ld, ld, tid);
    load_tile<HD, BQ, NT>(sO0 + buf * BQ * HD * 2, dOg + (long long)qb * BQ * ld_o, ld_o, tid);
    for (int i = tid; i < BQ; i += NT) {
      sL[buf * BQ + i] = Lg[qb * BQ + i] * 1.4426950408889634f;
      sDv[buf * BQ + i] = Dg[qb * BQ + i];
    }
  };
  load_q(qb_begin, 0);
  cp_async_commit();

  uint32_t kf[KSTEPS][4], vf[KSTEPS][4];
  float dk[DT][4], dv[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }

  for (int qb = qb_begin; qb < nqb; ++qb) {
    const int buf = (qb - qb_begin) & 1;
    __syncthreads();  // previous iteration finished reading the other buffers / sdS
    if (qb + 1 < nqb) {
      load_q(qb + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (qb == qb_begin) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sK + tile_off<HD>(r, c), kf[kk][0], kf[kk][1], kf[kk][2], kf[kk][3]);
        ldsm_x4(sV + tile_off<HD>(r, c), vf[kk][0], vf[kk][1], vf[kk][2], vf[kk][3]);
      }
    }
    const uint32_t sQ = sQ0 + buf * BQ * HD * 2;
    const uint32_t sO = sO0 + buf * BQ * HD * 2;
    const float* L = sL + buf * BQ;
    const float* Dv = sDv + buf * BQ;
    // S^T = K Q^T and dP^T = V dO^T : 16 keys x 64 queries per warp
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
      dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int idx = lane >> 3;
        const int r = np * 16 + (idx >> 1) * 8 + (lane & 7);
        const int c = kk * 2 + (idx & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sQ + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(st[2 * np], kf[kk][0], kf[kk][1], kf[kk][2], kf[kk][3], b0, b1);
        mma16816(st[2 * np + 1], kf[kk][0], kf[kk][1], kf[kk][2], kf[kk][3], b2, b3);
        ldsm_x4(sO + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(dpt[2 * np], vf[kk][0], vf[kk][1], vf[kk][2], vf[kk][3], b0, b1);
        mma16816(dpt[2 * np + 1], vf[kk][0], vf[kk][1], vf[kk][2], vf[kk][3], b2, b3);
      }
    }
    // P^T and dS^T
    const int key0 = k0 + warp * 16 + g, key1 = key0 + 8;
    const int qbase = qb * BQ;
    uint32_t pa[4][4], da[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int ql = nt * 8 + 2 * t;  // local query index of element 0
      const int q = qbase + ql;
      float p[4], ds[4];
      const float lq0 = L[ql], lq1 = L[ql + 1];
      p[0] = (key0 <= q) ? exp2f(st[nt][0] * sl2 - lq0) : 0.f;
      p[1] = (key0 <= q + 1) ? exp2f(st[nt][1] * sl2 - lq1) : 0.f;
      p[2] = (key1 <= q) ? exp2f(st[nt][2] * sl2 - lq0) : 0.f;
      p[3] = (key1 <= q + 1) ? exp2f(st[nt][3] * sl2 - lq1) : 0.f;
      const float d0 = Dv[ql], d1 = Dv[ql + 1];
      ds[0] = p[0] * (dpt[nt][0] - d0);
      ds[1] = p[1] * (dpt[nt][1] - d1);
      ds[2] = p[2] * (dpt[nt][2] - d0);
      ds[3] = p[3] * (dpt[nt][3] - d1);
      const int kk = nt >> 1, hi = nt & 1;
      pa[kk][hi * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[kk][hi * 2 + 1] = pack_bf16x2(p[2], p[3]);
      da[kk][hi * 2 + 0] = pack_bf16x2(ds[0], ds[1]);
      da[kk][hi * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
      // dS[q][key] into smem (transposed store) for the dQ product
      const int kl0 = warp * 16 + g, kl1 = kl0 + 8;
      uint16_t* sds = reinterpret_cast<uint16_t*>(smem + (sdS - sK));
      auto put = [&](int qq, int kl, float v) {
        const uint32_t off = tile_off<64>(qq, kl >> 3) + (kl & 7) * 2;
        __nv_bfloat16 hv = __float2bfloat16_rn(v);
        sds[off >> 1] = *reinterpret_cast<uint16_t*>(&hv);
      };
      put(ql, kl0, ds[0]);
      put(ql + 1, kl0, ds[1]);
      put(ql, kl1, ds[2]);
      put(ql + 1, kl1, ds[3]);
    }
    // dV += P^T dO ; dK += dS^T Q      (B operands: dO / Q row-major -> transposed ldmatrix)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int idx = lane >> 3;
        const int r = kk * 16 + (idx & 1) * 8 + (lane & 7);
        const int c = dp * 2 + (idx >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sO + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(dv[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma16816(dv[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
        ldsm_x4_t(sQ + tile_off<HD>(r, c), b0, b1, b2, b3);
        mma16816(dk[2 * dp], da[kk][0], da[kk][1], da[kk][2], da[kk][3], b0, b1);
        mma16816(dk[2 * dp + 1], da[kk][0], da[kk][1], da[kk][2], da[kk][3], b2, b3);
      }
    }
    __syncthreads();  // sdS complete
    // dQ[q, d] += scale * sum_key dS[q,key] K[key,d]   (warp w: queries 16w..16w+15)
    {
      float dq[DT][4];
#pragma unroll
      for (int i = 0; i < DT; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 64 keys
        uint32_t a0, a1, a2, a3;
        {
          const int r = warp * 16 + (lane & 15);
          const int c = kk * 2 + (lane >> 4);
          ldsm_x4(sdS + tile_off<64>(r, c), a0, a1, a2, a3);
        }
#pragma unroll
        for (int dp = 0; dp < HD / 16; ++dp) {
          const int idx = lane >> 3;
          const int r = kk * 16 + (idx & 1) * 8 + (lane & 7);
          const int c = dp * 2 + (idx >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sK + tile_off<HD>(r, c), b0, b1, b2, b3);
          mma16816(dq[2 * dp], a0, a1, a2, a3, b0, b1);
          mma16816(dq[2 * dp + 1], a0, a1, a2, a3, b2, b3);
        }
      }
      const int q0r = qbase + warp * 16 + g;
      float* dq0 = dq_acc + (row0 + q0r) * (long long)D + h * HD;
      float* dq1 = dq0 + 8 * (long long)D;
#pragma unroll
      for (int dt = 0; dt < DT; ++dt) {
        const int c = dt * 8 + 2 * t;
        atomicAdd(reinterpret_cast<float2*>(dq0 + c), make_float2(dq[dt][0] * scale, dq[dt][1] * scale));
        atomicAdd(reinterpret_cast<float2*>(dq1 + c), make_float2(dq[dt][2] * scale, dq[dt][3] * scale));
      }
    }
  }
  // write dK (scaled) and dV into the fused gradient buffer
  const int kr0 = k0 + warp * 16 + g;
  __nv_bfloat16* dk0 = dqkv + (row0 + kr0) * ld_d + D + h * HD;
  __nv_bfloat16* dk1 = dk0 + 8 * ld_d;
  __nv_bfloat16* dv0 = dqkv + (row0 + kr0) * ld_d + 2 * D + h * HD;
  __nv_bfloat16* dv1 = dv0 + 8 * ld_d;
#pragma unroll
  for (int dt = 0; dt < DT; ++dt) {
    const int c = dt * 8 + 2 * t;
    float a0 = dk[dt][0] * scale, a1 = dk[dt][1] * scale, a2 = dk[dt][2] * scale, a3 = dk[dt][3] * scale;
    if (rope_cs != nullptr) {  // k was rotated by +theta in the forward: rotate its gradient by -theta
      const float2 r0 = rope_cs[kr0 * (HD / 2) + (c >> 1)];
      const float2 r1 = rope_cs[(kr0 + 8) * (HD / 2) + (c >> 1)];
      const float b0 = a0 * r0.x + a1 * r0.y, b1 = -a0 * r0.y + a1 * r0.x;
      const float b2 = a2 * r1.x + a3 * r1.y, b3 = -a2 * r1.y + a3 * r1.x;
      a0 = b0; a1 = b1; a2 = b2; a3 = b3;
    }
    *reinterpret_cast<uint32_t*>(dk0 + c) = pack_bf16x2(a0, a1);
    *reinterpret_cast<uint32_t*>(dk1 + c) = pack_bf16x2(a2, a3);
    *reinterpret_cast<uint32_t*>(dv0 + c) = pack_bf16x2(dv[dt][0], dv[dt][1]);
    *reinterpret_cast<uint32_t*>(dv1 + c) = pack_bf16x2(dv[dt][2], dv[dt][3]);
  }
}

// dqkv[:, 0:D] = bf16(dq_acc), optionally rotated by -theta (RoPE backward of q)
__global__ void attn_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv,
                                       long long ld_d, long long M, int D, int S, int HD,
                                       const float2* __restrict__ rope_cs) {
  const long long total = M * (D / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (D / 2);
    const int c = (int)(i % (D / 2)) * 2;
    float2 v = *reinterpret_cast<const float2*>(dq_acc + r * D + c);
    if (rope_cs != nullptr) {
      const float2 cs = rope_cs[(int)(r % S) * (HD / 2) + ((c % HD) >> 1)];
      v = make_float2(v.x * cs.x + v.y * cs.y, -v.x * cs.y + v.y * cs.x);
    }
    *reinterpret_cast<uint32_t*>(dqkv + r * ld_d + c) = pack_bf16x2(v.x, v.y);
  }
}

}  // namespace attn
}  // namespace pcb

using namespace pcb;
using namespace pcb::attn;

template <int HD, int NW>
static int fwd_launch(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                      float scale, cudaStream_t s) {
  constexpr int BQ = 16 * NW;
  const size_t smem = (size_t)(BQ * HD * 2 + 4 * 64 * HD * 2);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_fwd_kernel<HD, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  dim3 grid(S / BQ, B * H);
  attn_fwd_kernel<HD, NW><<<grid, NW * 32, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(qkv), ld,
                                                       reinterpret_cast<__nv_bfloat16*>(out), ld_o, lse, S, H, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int pcb_attn_fwd(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H, int HD,
                 float scale, cudaStream_t s) {
  if (S % 128 != 0 || ld % 8 || ld_o % 8) return -1;
  if (HD == 64) return fwd_launch<64, 8>(qkv, ld, out, ld_o, lse, B, S, H, scale, s);
  if (HD == 128) return fwd_launch<128, 8>(qkv, ld, out, ld_o, lse, B, S, H, scale, s);
  return -1;
}

template <int HD>
static int bwd_launch(const void* qkv, long long ld, const void* dout, long long ld_o, const float* lse,
                      const float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H, float scale,
                      const float* rope_cs, cudaStream_t s) {
  const size_t smem = (size_t)(2 * 64 * HD * 2 + 4 * 64 * HD * 2 + 64 * 64 * 2 + 4 * 64 * 4);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  dim3 grid(S / 64, B * H);
  attn_bwd_kernel<HD><<<grid, 128, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(qkv), ld,
                                              reinterpret_cast<const __nv_bfloat16*>(dout), ld_o, lse, dvec, dq_acc,
                                              reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d, S, H, scale,
                                              reinterpret_cast<const float2*>(rope_cs));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// Full attention backward: preprocess, main kernel, dQ conversion.  dq_acc [B*S, D] fp32 and
// dvec [B*H, S] fp32 are scratch.
// Same as pcb_attn_bwd, and when rope_cs is given (cos/sin table [S][HD/2]) the dq and dk it writes are
// already rotated back by -theta, i.e. they are gradients w.r.t. the pre-RoPE q and k.
int pcb_attn_bwd_rope(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                      const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                      int HD, float scale, const float* rope_cs, cudaStream_t s) {
  if (S % 128 != 0 || ld % 8 || ld_o % 8 || ld_d % 8) return -1;
  const long long rows = (long long)B * S * H;
  attn_bwd_pre_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(out),
                                                                  reinterpret_cast<const __nv_bfloat16*>(dout), ld_o,
                                                                  dvec, dq_acc, B, S, H, HD);
  if (cudaGetLastError() != cudaSuccess) return -3;
  int r;
  if (HD == 64) r = bwd_launch<64>(qkv, ld, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, scale, rope_cs, s);
  else if (HD == 128)
    r = bwd_launch<128>(qkv, ld, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, scale, rope_cs, s);
  else return -1;
  if (r) return r;
  const long long total = (long long)B * S * (H * HD / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  attn_dq_convert_kernel<<<(unsigned)blocks, 256, 0, s>>>(dq_acc, reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d,
                                                          (long long)B * S, H * HD, S, HD,
                                                          reinterpret_cast<const float2*>(rope_cs));
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// The two helper passes of the backward, shared with the tcgen05 main kernel (attention_bwd_tc.cu).
int pcb_attn_bwd_pre(const void* out, const void* dout, long long ld_o, float* dvec, float* dq_acc, int B, int S,
                     int H, int HD, cudaStream_t s) {
  const long long rows = (long long)B * S * H;
  attn_bwd_pre_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(out),
                                                                  reinterpret_cast<const __nv_bfloat16*>(dout), ld_o,
                                                                  dvec, dq_acc, B, S, H, HD);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(1000 + static_cast<int>(e));
}

int pcb_attn_dq_convert(const float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H, int HD,
                        const float* rope_cs, cudaStream_t s) {
  const long long total = (long long)B * S * (H * HD / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  attn_dq_convert_kernel<<<(unsigned)blocks, 256, 0, s>>>(dq_acc, reinterpret_cast<__nv_bfloat16*>(dqkv), ld_d,
                                                          (long long)B * S, H * HD, S, HD,
                                                          reinterpret_cast<const float2*>(rope_cs));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -(1000 + static_cast<int>(e));
}

int pcb_attn_bwd(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o, const float* lse,
                 float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H, int HD, float scale,
                 cudaStream_t s) {
  return pcb_attn_bwd_rope(qkv, ld, out, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, HD, scale, nullptr, s);
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant (see attention_noalloc.h for who needs it and the contract).
// Same kernels as the regular backward (tcgen05 for head dim 64, the mma.sync kernels for 128);
// the two fp32 scratch buffers come from a file-scope device array instead of the caller.
// ------------------------------------------------------------------------------------------
#include <cstdio>
#include <mutex>

#include "attention_noalloc.h"

int pcb_attn_bwd_tc(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                    const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                    int HD, float scale, const float* rope_cs, int* err, cudaStream_t s);

namespace {

constexpr size_t kNoAllocFloats = PCB_ATTN_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_attn_bwd_scratch[kNoAllocFloats];

constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
float* g_noalloc_base[kMaxDevices] = {};

// Device address of g_attn_bwd_scratch on the current device, looked up once per device.
// The symbol name is only a host-side handle; the address must come from the runtime.
int noalloc_scratch(float** base) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -8;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_base[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      fprintf(stderr, "pcb_attn_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
              cudaGetErrorString(e));
      return -9;
    }
    g_noalloc_base[dev] = static_cast<float*>(p);
  }
  *base = g_noalloc_base[dev];
  return 0;
}

// Scratch floats the problem needs: the dQ accumulator (rounded up to 64 floats, so the row
// dot-products that follow it start on a 256-byte boundary) plus B*H*S row dot-products.
// Returns false when a product overflows 64 bits; the caller treats that as "too large".
bool noalloc_need(int B, int S, int H, int HD, size_t* dq_floats, size_t* need) {
  size_t bs, bsh, bshd, bhs;
  if (__builtin_mul_overflow((size_t)B, (size_t)S, &bs) || __builtin_mul_overflow(bs, (size_t)H, &bsh) ||
      __builtin_mul_overflow(bsh, (size_t)HD, &bshd) || bshd > SIZE_MAX - 63)
    return false;
  bhs = bsh;  // B*H*S
  *dq_floats = (bshd + 63) / 64 * 64;
  if (*dq_floats > SIZE_MAX - bhs) return false;
  *need = *dq_floats + bhs;
  return true;
}

}  // namespace

extern "C" int pcb_attn_bwd_noalloc(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                                    const float* lse, void* dqkv, long long ld_d, int B, int S, int H, int HD,
                                    float scale, cudaStream_t s) {
  if (B <= 0 || H <= 0 || S <= 0 || S % 128 != 0 || ld % 8 || ld_o % 8 || ld_d % 8) return -1;
  if (HD != 64 && HD != 128) return -1;
  size_t dq_floats = 0, need = 0;
  if (!noalloc_need(B, S, H, HD, &dq_floats, &need) || need > kNoAllocFloats) {
    fprintf(stderr,
            "pcb_attn_bwd_noalloc: problem B=%d S=%d H=%d HD=%d needs more than the built-in scratch of %zu "
            "floats (%u bytes); use pcb_attn_bwd with caller-provided buffers\n",
            B, S, H, HD, kNoAllocFloats, (unsigned)PCB_ATTN_NOALLOC_SCRATCH_BYTES);
    return PCB_ATTN_NOALLOC_E_TOO_LARGE;
  }
  // tensor-core loads and 16-byte vector stores need every operand on a 16-byte boundary
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(dout) |
       reinterpret_cast<uintptr_t>(lse) | reinterpret_cast<uintptr_t>(dqkv)) & 15)
    return PCB_ATTN_NOALLOC_E_ALIGN;
  float* base = nullptr;
  const int rc = noalloc_scratch(&base);
  if (rc != 0) return rc;
  float* dq_acc = base;
  float* dvec = base + dq_floats;
  // both paths clear dq_acc before accumulating, so an earlier call's partial sums never leak in
  if (HD == 64) {
    const int r = pcb_attn_bwd_tc(qkv, ld, out, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, HD, scale,
                                  nullptr, nullptr, s);
    return r <= -1000 ? -3 : r;
  }
  return pcb_attn_bwd(qkv, ld, out, dout, ld_o, lse, dvec, dq_acc, dqkv, ld_d, B, S, H, HD, scale, s);
}
