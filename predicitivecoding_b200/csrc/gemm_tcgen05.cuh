// tcgen05 / TMEM / TMA GEMM for sm_100a with fused epilogues.
//
//   C[M,N] = epilogue( A[M,K] * B[K,N] ),  bf16 operands, fp32 accumulation.
//
// Each operand is either K-major (rows of K contiguous) or MN-major (rows of M/N
// contiguous).  All three products of a linear layer map onto it without any
// transpose kernel:  Y = X W^T (A K-major, B K-major),  dX = dY W (A K-major,
// B N-major) and  dW = dY^T X (A M-major, B N-major).
//
// Design: persistent kernel, one CTA per SM, 6 warps:
//   warp 0       TMA producer (one elected lane), multi-stage smem ring
//   warp 1       TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..5   epilogue: tcgen05.ld of the accumulator, fused math, stores
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.  Split-K is supported
// for the reductions over tokens (weight gradients), using vector fp32 atomics.
//
// Parity notes (reference behaviour the epilogues reproduce):
//   * GELU is the tanh form with 0.7978845608 / 0.044715
//     (PredictiveCoding.LLM/Autograd/Autograd.cs:303-328).
//   * "beta = 1" residual GEMMs of DeviceDecoderTrainer
//     (PredictiveCoding.Device/Training/DeviceDecoderTrainer.cs:410-433) become EPI_ACC_F32.
//   * The PC epilogues restate Layer.ComputePrediction / SetPredictionError /
//     UpdateState / UpdateWeights (PredicitiveCoding/Model/Layer.cs:212-333) over a batch,
//     as BatchedPcForward does on the host (PredictiveCoding.Device/BatchedPcForward.cs:74-128).
#pragma once

#include "common.cuh"
#include "gemm_api.h"

