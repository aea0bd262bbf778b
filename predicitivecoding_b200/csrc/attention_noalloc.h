// Allocation-free entry point of the causal attention backward.
//
// Declaration note: this entry point has no counterpart in the reference project
// (matteofabbri/PredicitiveCoding); it exists only in this library.
//
// Who it is for.  The regular backward (pcb_attn_bwd) needs two fp32 scratch
// buffers -- the dQ accumulator [B*S, H*HD] and the row dot-products dO.O
// [B*H, S] -- and expects the caller to allocate them.  Some callers cannot
// allocate device memory at the point where they call attention: a host that
// manages every byte of device memory through its own pool and forbids
// cudaMalloc, a latency-critical loop that must not take the implicit device
// synchronisation cudaMalloc/cudaFree can cause, or a foreign-language host
// that reaches this library only through a C ABI and has no CUDA allocator of
// its own.  pcb_attn_bwd_noalloc serves them: the caller passes only the
// inputs and the output, and the scratch lives in a fixed device array inside
// this library.
//
// Contract.
//   * Scratch is a file-scope __device__ array of PCB_ATTN_NOALLOC_SCRATCH_BYTES
//     (16 MiB).  Every GPU that loads this library holds that memory until the
//     process exits.
//   * Capacity: B*S*H*HD (rounded up to 64) + B*H*S floats must fit in the
//     array.  Larger problems are rejected with PCB_ATTN_NOALLOC_E_TOO_LARGE and
//     a message on stderr; nothing is launched.
//   * Set-up: the first call on each device, with that device current, looks up
//     the array's device address (cudaGetSymbolAddress) and caches it for that
//     device.  Make that first call on a device before any stream capture on it.
//     The cached address belongs to the device's primary context: after
//     cudaDeviceReset (or any teardown of that context) it is stale and the
//     process must not call this entry point on that device again.
//   * No allocation: the call performs no cudaMalloc, cudaFree or allocating
//     library call.
//   * Shared state: every call uses the same array, which keeps the previous
//     call's contents; the call clears the dQ accumulator itself before use.
//     Calls whose GPU work overlaps (different streams, or different host
//     threads on one device) race on the array and corrupt each other's
//     results: serialise them.
//   * Inputs/outputs are exactly those of pcb_attn_bwd: qkv [B*S, ld] bf16
//     (q | k | v at column offsets 0, H*HD, 2*H*HD), out and dout [B*S, ld_o]
//     bf16, lse [B*H, S] fp32 from the forward; dqkv [B*S, ld_d] bf16 receives
//     dq | dk | dv.  S must be a multiple of 128 and HD 64 or 128; qkv, out,
//     dout, lse and dqkv must start on 16-byte boundaries and every row stride
//     must be a multiple of 8 elements.  Head dim 64 runs the tcgen05 backward,
//     head dim 128 the mma.sync backward, exactly as the regular entry point.
//   * Size arithmetic is overflow-checked: shapes whose element counts do not
//     fit in 64 bits are rejected like any other oversized problem.
//
// Return codes: 0 success; -1 unsupported shape/stride; -3 launch failure;
// -5 tensor-map encoding failed; PCB_ATTN_NOALLOC_E_TOO_LARGE (-7) scratch too
// small; -8 no current device; -9 the scratch address lookup failed;
// PCB_ATTN_NOALLOC_E_ALIGN (-10) an operand is not 16-byte aligned.
#pragma once

#include <cuda_runtime.h>

#define PCB_ATTN_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
#define PCB_ATTN_NOALLOC_E_TOO_LARGE (-7)
#define PCB_ATTN_NOALLOC_E_ALIGN (-10)

#ifdef __cplusplus
extern "C" {
#endif

int pcb_attn_bwd_noalloc(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                         const float* lse, void* dqkv, long long ld_d, int B, int S, int H, int HD, float scale,
                         cudaStream_t stream);

#ifdef __cplusplus
}
#endif
