// Host-side interface of the skinny decode GEMM's RoPE + KV-cache append epilogue.
#pragma once

#include <cuda_bf16.h>

struct SkinnyRope {
  __nv_bfloat16* q;        // [M, heads * hd] rotated queries
  __nv_bfloat16* k;        // [M, heads, cap, hd] key cache (row *pos written)
  __nv_bfloat16* v;        // [M, heads, cap, hd] value cache (row *pos written)
  const float* cs;         // [cap, hd / 2, 2] cos / sin
  const long long* pos;    // device scalar: the position of this token
  int heads, hd, cap;
};
