// Epilogue math shared by the 1-CTA and 2-CTA tcgen05 GEMM kernels: one 32-column
// accumulator chunk of one row (a TMEM lane) is transformed and stored per call.
#pragma once

#include "gemm_tcgen05.cuh"

namespace pcb {

PCB_DEVICE float act_apply(int act, float x) {
  switch (act) {
    case 1: return tanhf(x);
    case 2: return fmaxf(x, 0.f);
    case 3: return 1.f / (1.f + __expf(-x));
    default: return x;
  }
}
// derivative from pre-activation x and activation y (tanh/sigmoid use y as the reference does)
PCB_DEVICE float act_deriv(int act, float x, float y) {
  switch (act) {
    case 1: return 1.f - y * y;
    case 2: return x > 0.f ? 1.f : 0.f;
    case 3: return y * (1.f - y);
    default: return 1.f;
  }
}

PCB_DEVICE void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u;
      u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      d4[j] = u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

PCB_DEVICE void load_bf16x32(const __nv_bfloat16* src, float (&v)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u = s4[j];
      v[8 * j + 0] = bf16_lo(u.x); v[8 * j + 1] = bf16_hi(u.x);
      v[8 * j + 2] = bf16_lo(u.y); v[8 * j + 3] = bf16_hi(u.y);
      v[8 * j + 4] = bf16_lo(u.z); v[8 * j + 5] = bf16_hi(u.z);
      v[8 * j + 6] = bf16_lo(u.w); v[8 * j + 7] = bf16_hi(u.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < nvalid) ? __bfloat162float(src[j]) : 0.f;
  }
}

PCB_DEVICE void load_f32x32(const float* src, float (&v)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 f = s4[j];
      v[4 * j + 0] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < nvalid) ? src[j] : 0.f;
  }
}

PCB_DEVICE void store_f32x32(float* dst, const float (&v)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) dst[j] = v[j];
  }
}

PCB_DEVICE void red_f32x32(float* dst, const float (&v)[32], int nvalid) {
  if (nvalid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(d4 + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) atomicAdd(dst + j, v[j]);
  }
}

PCB_DEVICE void tmem_load_f32x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// One 32-column chunk of a "plain" epilogue (everything except the SwiGLU pairs).
template <int EPI>
PCB_DEVICE void epilogue_chunk(const GemmArgs& a, int m, int n, float (&v)[32], bool row_ok, long long boff = 0) {
  const int nvalid = min(32, a.N - n);
  if (!row_ok || nvalid <= 0) return;
  if (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_ACC_F32 || EPI == EPI_GELU || EPI == EPI_RESID_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
    if (a.bias != nullptr) {
      float b[32];
      if (a.bias_bf16) load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(a.bias) + boff + n, b, nvalid);
      else load_f32x32(reinterpret_cast<const float*>(a.bias) + boff + n, b, nvalid);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += b[j];
    }
  }
  if (EPI == EPI_RS_BF16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
    const int c = m / a.rs_rows;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.rs_peers[c]) +
                         (long long)(a.rs_rank * a.rs_rows + (m - c * a.rs_rows)) * a.ldc + n;
    store_bf16x32(dst, v, nvalid);   // plain stores into the owner's slot over NVLink
    return;
  }
  if (EPI == EPI_BF16) {
    if (a.rope_cs != nullptr && n < a.rope_cols) {
      const float2* cs = reinterpret_cast<const float2*>(a.rope_cs) + (long long)(m % a.rope_S) * (a.rope_hd >> 1);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 c = cs[((n + j) % a.rope_hd) >> 1];
        const float x0 = v[j], x1 = v[j + 1];
        v[j] = x0 * c.x - x1 * c.y;
        v[j + 1] = x0 * c.y + x1 * c.x;
      }
    }
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_F32) {
    store_f32x32(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_ACC_F32) {
    float* c = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    float o[32];
    load_f32x32(c, o, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] += v[j];
    store_f32x32(c, o, nvalid);
  } else if (EPI == EPI_RESID_F32) {
    float r[32];
    load_f32x32(reinterpret_cast<const float*>(a.aux) + (long long)m * a.ldaux + n, r, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += r[j];
    store_f32x32(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_RED_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= a.alpha;
    red_f32x32(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_GELU) {
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
    float g[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) g[j] = gelu_tanh_fast(__bfloat162float(__float2bfloat16_rn(v[j])));
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, g, nvalid);
  } else if (EPI == EPI_GELU_BWD) {
    float p[32];
    load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(a.aux) + (long long)m * a.ldaux + n, p, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = a.alpha * v[j] * gelu_tanh_grad_fast(p[j]);
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_SWIGLU_BWD) {
    // n indexes the activation columns f; 32 | 64 so a chunk stays inside one group
    const int grp = n >> 6, off = n & 63;
    const long long gcol = (long long)grp * 128 + off;
    const __nv_bfloat16* pre = reinterpret_cast<const __nv_bfloat16*>(a.aux) + (long long)m * a.ldaux;
    float g[32], u[32];
    load_bf16x32(pre + gcol, g, nvalid);
    load_bf16x32(pre + gcol + 64, u, nvalid);
    float dg[32], du[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float dh = a.alpha * v[j];
      const float s = __fdividef(1.f, 1.f + __expf(-g[j]));
      const float silu = g[j] * s;
      du[j] = dh * silu;
      dg[j] = dh * u[j] * s * (1.f + g[j] * (1.f - s));
    }
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc;
    store_bf16x32(out + gcol, dg, nvalid);
    store_bf16x32(out + gcol + 64, du, nvalid);
  } else if (EPI == EPI_BF16_ACC) {
    float r[32];
    load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(a.aux) + (long long)m * a.ldaux + n, r, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = a.alpha * v[j] + r[j];
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nvalid);
  } else if (EPI == EPI_PC_PRED) {
    float b[32];
    if (a.bias != nullptr) load_f32x32(reinterpret_cast<const float*>(a.bias) + n, b, nvalid);
    else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = 0.f;
    }
    float pre[32], pred[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      pre[j] = v[j] + b[j];
      pred[j] = act_apply(a.act, pre[j]);
    }
    if (a.pc_pred_out != nullptr)
      store_f32x32(reinterpret_cast<float*>(a.pc_pred_out) + (long long)m * a.ld_pred + n, pred, nvalid);
    if (a.pc_pred_bf16 != nullptr)
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.pc_pred_bf16) + (long long)m * a.ld_pred + n, pred, nvalid);
    if (a.C != nullptr) {
      float mb[32];
      load_f32x32(reinterpret_cast<const float*>(a.aux) + (long long)m * a.ldaux + n, mb, nvalid);
      float e[32], dl[32];
      float sq = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        e[j] = a.pc_pi * (mb[j] - pred[j]);
        dl[j] = act_deriv(a.act, pre[j], pred[j]) * e[j];
        if (j < nvalid) sq += e[j] * e[j];
      }
      store_f32x32(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, e, nvalid);
      if (a.D != nullptr)
        store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, dl, nvalid);
      if (a.pc_energy != nullptr) atomicAdd(a.pc_energy, sq);
    }
  } else if (EPI == EPI_PC_STATE) {
    float* mu = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    float s[32], e[32];
    load_f32x32(mu, s, nvalid);
    if (a.aux != nullptr) load_f32x32(reinterpret_cast<const float*>(a.aux) + (long long)m * a.ldaux + n, e, nvalid);
    else {
#pragma unroll
      for (int j = 0; j < 32; ++j) e[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float grad = e[j] - v[j];
      if (a.pc_actreg > 0.f) grad += a.pc_actreg * (s[j] > 0.f ? 1.f : (s[j] < 0.f ? -1.f : 0.f));
      s[j] -= a.pc_eta * grad;
    }
    store_f32x32(mu, s, nvalid);
    if (a.D != nullptr)
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, s, nvalid);
  } else if (EPI == EPI_PC_WUPD) {
    float* w = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    float x[32];
    load_f32x32(w, x, nvalid);
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = (x[j] + a.alpha * v[j]) * a.pc_decay;
    store_f32x32(w, x, nvalid);
    if (a.D != nullptr)
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, x, nvalid);
  }
}


// ---------------------------------------------------------------------------------------------
// Coalesced epilogue: the same transformations, applied to 4 consecutive columns of one row by one
// lane after the warp has transposed its 32x32 accumulator chunk through shared memory, so that 8
// lanes cover one 128-byte row segment and every global load / store instruction touches 4 full
// rows instead of 32 partial ones.  Returns this lane's squared-error contribution (EPI_PC_PRED).
// EPI_SWIGLU_BWD has a vec4 form too but measured slower than the row path (its gate / up halves
// are 64 columns apart), so it stays on the row path.
template <int EPI>
PCB_DEVICE constexpr bool epi_coalesced() {
  return EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_ACC_F32 || EPI == EPI_RESID_F32 || EPI == EPI_RED_F32 ||
         EPI == EPI_GELU || EPI == EPI_GELU_BWD || EPI == EPI_BF16_ACC || EPI == EPI_RS_BF16 ||
         EPI == EPI_PC_PRED || EPI == EPI_PC_STATE || EPI == EPI_PC_WUPD;
}

PCB_DEVICE bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
PCB_DEVICE bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

PCB_DEVICE void ld_f32x4(const float* p, float (&v)[4], int nv) {
  if (nv == 4 && al16(p)) {
    const float4 f = *reinterpret_cast<const float4*>(p);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = j < nv ? p[j] : 0.f;
  }
}
PCB_DEVICE void st_f32x4(float* p, const float (&v)[4], int nv) {
  if (nv == 4 && al16(p)) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < nv) p[j] = v[j];
  }
}
PCB_DEVICE void ld_bf16x4(const __nv_bfloat16* p, float (&v)[4], int nv) {
  if (nv == 4 && al8(p)) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = j < nv ? __bfloat162float(p[j]) : 0.f;
  }
}
PCB_DEVICE void st_bf16x4(__nv_bfloat16* p, const float (&v)[4], int nv) {
  if (nv == 4 && al8(p)) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < nv) p[j] = __float2bfloat16_rn(v[j]);
  }
}

// Everything a vec4 epilogue reads besides the accumulator and per-column vectors, issued for all
// of a chunk's rows before any of them is finished so the loads overlap (p[0..3], p[4..7]).
template <int EPI>
PCB_DEVICE void epi_prefetch(const GemmArgs& a, int m, int n, float (&p)[8], bool row_ok) {
  const int nv = min(4, a.N - n);
  if (!row_ok || nv <= 0) return;
  float* q0 = p;
  float (&lo)[4] = *reinterpret_cast<float(*)[4]>(q0);
  float (&hi)[4] = *reinterpret_cast<float(*)[4]>(q0 + 4);
  if (EPI == EPI_ACC_F32 || EPI == EPI_PC_STATE || EPI == EPI_PC_WUPD) {
    ld_f32x4(reinterpret_cast<const float*>(a.C) + (long long)m * a.ldc + n, lo, nv);
    if (EPI == EPI_PC_STATE) {
      if (a.aux != nullptr) ld_f32x4(reinterpret_cast<const float*>(a.aux) + (long long)m * a.ldaux + n, hi, nv);
      else {
#pragma unroll
        for (int j = 0; j < 4; ++j) hi[j] = 0.f;
      }
    }
  } else if (EPI == EPI_RESID_F32 || (EPI == EPI_PC_PRED)) {
    if (EPI == EPI_PC_PRED && a.C == nullptr) return;
    ld_f32x4(reinterpret_cast<const float*>(a.aux) + (long long)m * a.ldaux + n, lo, nv);
  } else if (EPI == EPI_GELU_BWD || EPI == EPI_BF16_ACC) {
    ld_bf16x4(reinterpret_cast<const __nv_bfloat16*>(a.aux) + (long long)m * a.ldaux + n, lo, nv);
  } else if (EPI == EPI_SWIGLU_BWD) {
    const long long gcol = (long long)(n >> 6) * 128 + (n & 63);
    const __nv_bfloat16* pre = reinterpret_cast<const __nv_bfloat16*>(a.aux) + (long long)m * a.ldaux;
    ld_bf16x4(pre + gcol, lo, nv);
    ld_bf16x4(pre + gcol + 64, hi, nv);
  }
}

template <int EPI>
PCB_DEVICE float epilogue_vec4(const GemmArgs& a, int m, int n, float (&v)[4], const float (&p)[8], bool row_ok,
                                long long boff = 0) {
  const int nv = min(4, a.N - n);
  if (!row_ok || nv <= 0) return 0.f;
  if (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_ACC_F32 || EPI == EPI_GELU || EPI == EPI_RESID_F32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= a.alpha;
    if (a.bias != nullptr) {
      float b[4];
      if (a.bias_bf16) ld_bf16x4(reinterpret_cast<const __nv_bfloat16*>(a.bias) + boff + n, b, nv);
      else ld_f32x4(reinterpret_cast<const float*>(a.bias) + boff + n, b, nv);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] += b[j];
    }
  }
  if (EPI == EPI_BF16) {
    if (a.rope_cs != nullptr && n < a.rope_cols) {
      const float2* cs = reinterpret_cast<const float2*>(a.rope_cs) + (long long)(m % a.rope_S) * (a.rope_hd >> 1);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        const float2 c = cs[((n + j) % a.rope_hd) >> 1];
        const float x0 = v[j], x1 = v[j + 1];
        v[j] = x0 * c.x - x1 * c.y;
        v[j + 1] = x0 * c.y + x1 * c.x;
      }
    }
    st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nv);
  } else if (EPI == EPI_F32) {
    st_f32x4(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, v, nv);
  } else if (EPI == EPI_RS_BF16) {
    // row m goes to slot rs_rank of its owner c = m / rs_rows (plain 8-byte stores, over NVLink when remote)
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= a.alpha;
    const int c = m / a.rs_rows;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.rs_peers[c]) +
                         (long long)(a.rs_rank * a.rs_rows + (m - c * a.rs_rows)) * a.ldc + n;
    st_bf16x4(dst, v, nv);
  } else if (EPI == EPI_ACC_F32) {
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = p[j] + v[j];
    st_f32x4(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, o, nv);
  } else if (EPI == EPI_RESID_F32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] += p[j];
    st_f32x4(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, v, nv);
  } else if (EPI == EPI_RED_F32) {
    float* c = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    if (nv == 4 && al16(c)) {
      atomicAdd(reinterpret_cast<float4*>(c), make_float4(a.alpha * v[0], a.alpha * v[1], a.alpha * v[2], a.alpha * v[3]));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < nv) atomicAdd(c + j, a.alpha * v[j]);
    }
  } else if (EPI == EPI_GELU) {
    st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nv);
    float g[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) g[j] = gelu_tanh_fast(__bfloat162float(__float2bfloat16_rn(v[j])));
    st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, g, nv);
  } else if (EPI == EPI_GELU_BWD) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = a.alpha * v[j] * gelu_tanh_grad_fast(p[j]);
    st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nv);
  } else if (EPI == EPI_SWIGLU_BWD) {
    const int grp = n >> 6, off = n & 63;
    const long long gcol = (long long)grp * 128 + off;
    float dg[4], du[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g = p[j], u = p[4 + j];
      const float dh = a.alpha * v[j];
      const float s = __fdividef(1.f, 1.f + __expf(-g));
      du[j] = dh * g * s;
      dg[j] = dh * u * s * (1.f + g * (1.f - s));
    }
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc;
    st_bf16x4(out + gcol, dg, nv);
    st_bf16x4(out + gcol + 64, du, nv);
  } else if (EPI == EPI_BF16_ACC) {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = a.alpha * v[j] + p[j];
    st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.C) + (long long)m * a.ldc + n, v, nv);
  } else if (EPI == EPI_PC_PRED) {
    float b[4] = {0.f, 0.f, 0.f, 0.f};
    if (a.bias != nullptr) ld_f32x4(reinterpret_cast<const float*>(a.bias) + n, b, nv);
    float pre[4], pred[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pre[j] = v[j] + b[j];
      pred[j] = act_apply(a.act, pre[j]);
    }
    if (a.pc_pred_out != nullptr)
      st_f32x4(reinterpret_cast<float*>(a.pc_pred_out) + (long long)m * a.ld_pred + n, pred, nv);
    if (a.pc_pred_bf16 != nullptr)
      st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.pc_pred_bf16) + (long long)m * a.ld_pred + n, pred, nv);
    float sq = 0.f;
    if (a.C != nullptr) {
      float e[4], dl[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        e[j] = a.pc_pi * (p[j] - pred[j]);
        dl[j] = act_deriv(a.act, pre[j], pred[j]) * e[j];
        if (j < nv) sq += e[j] * e[j];
      }
      st_f32x4(reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n, e, nv);
      if (a.D != nullptr) st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, dl, nv);
    }
    return sq;
  } else if (EPI == EPI_PC_STATE) {
    float* mu = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    float s[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = p[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float grad = p[4 + j] - v[j];
      if (a.pc_actreg > 0.f) grad += a.pc_actreg * (s[j] > 0.f ? 1.f : (s[j] < 0.f ? -1.f : 0.f));
      s[j] -= a.pc_eta * grad;
    }
    st_f32x4(mu, s, nv);
    if (a.D != nullptr) st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, s, nv);
  } else if (EPI == EPI_PC_WUPD) {
    float* w = reinterpret_cast<float*>(a.C) + (long long)m * a.ldc + n;
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = (p[j] + a.alpha * v[j]) * a.pc_decay;
    st_f32x4(w, x, nv);
    if (a.D != nullptr) st_bf16x4(reinterpret_cast<__nv_bfloat16*>(a.D) + (long long)m * a.ldd + n, x, nv);
  }
  return 0.f;
}

}  // namespace pcb
