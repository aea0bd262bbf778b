// Host-safe GEMM API shared by the CUDA sources and the C++ bindings.
#pragma once
#include <cuda_runtime.h>

namespace pcb {

enum GemmEpi : int {
  EPI_BF16 = 0,        // C(bf16)  = alpha*acc + bias
  EPI_F32 = 1,         // C(f32)   = alpha*acc + bias
  EPI_ACC_F32 = 2,     // C(f32)  += alpha*acc + bias          (plain read-modify-write)
  EPI_RED_F32 = 3,     // C(f32)  += alpha*acc                 (atomic: split-K / accumulate)
  EPI_GELU = 4,        // C(bf16)  = pre = acc + bias ; D(bf16) = gelu(pre)
  EPI_SWIGLU = 5,      // C(bf16)  = pre [M,2F] (64-col gate/up interleave) ; D(bf16) = silu(g)*u [M,F]
  EPI_SWIGLU_BWD = 6,  // acc = d(act)[M,F], aux = pre[M,2F] ; C(bf16) = d(pre)[M,2F]
  EPI_GELU_BWD = 7,    // acc = d(act), aux = pre(bf16) ; C(bf16) = d(act)*gelu'(pre)
  EPI_PC_PRED = 8,     // PC prediction + error + delta (see gemm_epilogue_pc)
  EPI_PC_STATE = 9,    // PC state update
  EPI_PC_WUPD = 10,    // PC Hebbian weight update (single rank)
  EPI_BF16_ACC = 11,   // C(bf16) = alpha*acc + aux(bf16)      (bf16 residual add)
  EPI_RESID_F32 = 12,  // C(f32)  = aux(f32) + alpha*acc + bias (residual stream: x_out = x_in + f(x))
  EPI_RS_BF16 = 13,    // reduce-scatter partials: row m goes to owner c = m / rs_rows, slot rs_rank of
                       // owner c's buffer rs_peers[c] ([world * rs_rows, N] bf16, row stride ldc)
  EPI_COUNT = 14,
};

struct GemmArgs {
  int M, N, K;
  int a_mn, b_mn;
  int splits;           // K splits (>= 1)
  int kb_per_split;     // k-blocks (of 64) per split
  float alpha;
  void* C;              // primary output (see epilogue)
  long long ldc;
  void* D;              // secondary output
  long long ldd;
  const void* aux;      // auxiliary input
  long long ldaux;
  const void* bias;     // [N] or nullptr (fp32, or bf16 when bias_bf16)
  int bias_bf16;
  int* err;             // device error word (may be nullptr)
  // predictive-coding epilogue parameters
  int act;              // 0 linear, 1 tanh, 2 relu, 3 sigmoid
  float pc_pi;          // precision of the layer below (EPI_PC_PRED)
  float pc_eta;         // state lr (EPI_PC_STATE) / weight lr / batch (EPI_PC_WUPD)
  float pc_actreg;      // L1 activity regularisation (EPI_PC_STATE)
  float pc_decay;       // multiplicative decay (EPI_PC_WUPD): W <- (W + eta*acc) * decay
  float* pc_energy;     // sum of squared errors accumulator (EPI_PC_PRED), may be nullptr
  void* pc_pred_out;    // optional prediction output fp32 (EPI_PC_PRED, FFG warm start)
  long long ld_pred;
  void* pc_pred_bf16;   // optional bf16 copy of the prediction (FFG warm start)
  // fused RoPE (EPI_BF16): rotate interleaved pairs of columns [0, rope_cols) by the angle table
  // cs[pos][hd/2] = (cos, sin), pos = row % rope_S, pair = (col % rope_hd) / 2
  const float* rope_cs;
  int rope_S;
  int rope_hd;
  int rope_cols;
  // fused all-gather of A (tensor parallel, CTA-pair kernel only): A is this rank's gathered buffer
  // [ag_world * ag_rows, K]; chunk c of it is copied in-kernel from ag_peers[c] (same layout on
  // every rank) before the tiles of chunk c are loaded; ag_ready[c] counts CTAs done copying c.
  const void* const* ag_peers;  // device table [ag_world] (nullptr: no gather)
  void* ag_local;               // this rank's gathered buffer (same memory as the A operand)
  unsigned int* ag_ready;       // device counters [ag_world], zero at launch
  int ag_rows;
  int ag_rank;
  int ag_world;
  // reduce-scatter epilogue (EPI_RS_BF16)
  void* const* rs_peers;        // device table [world] of owners' slot buffers
  int rs_rows;
  int rs_rank;
  // tile order of the CTA-pair kernel without a fused gather: 0 = row blocks vary fastest (concurrent
  // tiles share B tiles), 1 = column blocks vary fastest (concurrent tiles share A tiles)
  int n_fastest;
  // EPI_BF16 / EPI_SWIGLU on the CTA-pair kernel: 1 when the launcher built tensor maps of the outputs,
  // so the epilogue stages bf16 boxes in shared memory and writes them with TMA stores
  int c_tma;
  // grouped GEMM (CTA-pair kernel only; mixture-of-experts FFNs).  grp_seg[0..grp_count] are the row
  // offsets of the experts' segments in a token buffer sorted by expert, each a multiple of 256 (the
  // pair tile); grp_seg[grp_count] is the number of rows in use.
  //   grp_mode 1 (rows): the M rows are the sorted buffer; a 256-row tile belongs to the expert whose
  //     segment holds it and reads that expert's block of B (B's N coordinate + e * grp_b_off when B is
  //     K-major, its K coordinate + e * grp_b_off when MN-major) and bias (+ e * grp_bias_off); tiles
  //     past the rows in use are skipped
  //   grp_mode 2 (K): weight gradients; the output stacks grp_count blocks of grp_m rows, block e
  //     contracts over the rows of segment e only (A and B MN-major over the sorted buffer)
  const int* grp_seg;
  int grp_count;
  int grp_mode;
  int grp_m;
  long long grp_b_off;
  long long grp_bias_off;
};

// Pair-kernel cycle counters (builds with PCB_GEMM_STATS): copies 12 counters to `out` and clears them.
int pcb_gemm_pair_stats(unsigned long long* out);

}  // namespace pcb

// Host entry: launches the kernel for the given operands.  Returns 0 on success.
// `A`/`B` are bf16 device pointers.  lda/ldb are row strides in elements of the
// operand as stored (K-major: stride between M/N rows; MN-major: stride between K rows).
int pcb_gemm_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb,
                    int epi, pcb::GemmArgs args, int force_bn, int force_splits, int num_sms,
                    cudaStream_t stream);

// Grouped (mixture-of-experts) GEMM on the CTA-pair kernel: `args` carries the grp_* fields (see
// GemmArgs); M, N, K are per expert except M in mode 1 (the sorted buffer's capacity) and K in mode 2
// (likewise).  Returns 0 on success, -1 bad operands, -6 bad group description.
int pcb_gemm_grouped_launch(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb,
                            int epi, pcb::GemmArgs args, int num_sms, cudaStream_t stream);
