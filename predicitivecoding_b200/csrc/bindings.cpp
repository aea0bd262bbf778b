// Python bindings for the sm_100a kernels (torch extension, built in-tree).
//
// Every entry takes torch tensors, launches on the current CUDA stream (so the
// calls compose with torch streams and CUDA-graph capture) and raises on a bad
// argument or a launch error.  No entry point allocates device memory except
// where the docstring says so.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <pybind11/stl.h>

#include <atomic>
#include <stdexcept>

// Argument and launch checks raise std::invalid_argument (pybind11 turns it into ValueError).
// c10::Error is not thrown from this library: a c10::Error raised from this extension after CUDA
// initialisation crashed the interpreter on the GPU hosts, while plain std exceptions go through
// pybind11's own translator.
#define PCB_CHECK(cond, ...)                                                    \
  do {                                                                          \
    if (!(cond)) throw std::invalid_argument(c10::str(__VA_ARGS__));            \
  } while (0)

#include "gemm_api.h"
#include "skinny_api.h"

// launchers defined in the .cu files
int pcb_embed_fwd(const int* tok, const void* W, float* x, int M, int D, int V, cudaStream_t s);
int pcb_embed_bwd(const int* tok, const float* dx, float* dW, int M, int D, int V, cudaStream_t s);
int pcb_rmsnorm_fwd(const float* x, const void* g, void* y, float* inv, int M, int D, float eps, cudaStream_t s);
int pcb_rmsnorm_bwd(const float* dy, const float* x, const void* g, const float* inv, float* dx, void* dx16,
                    float* dg, int M, int D, int accumulate, int num_sms, cudaStream_t s);
int pcb_rope(void* buf, long long ld, const float* cs, int M, int S, int D, int hd, int nparts, float sign,
             cudaStream_t s);
int pcb_ce(void* logits, long long ld, const int* tgt, float* loss, int M, int V, float scale, int write_grad,
           cudaStream_t s);
int pcb_sumsq(const float* x, long long n, float* out, int square, cudaStream_t s);
int pcb_colsum(const void* x, int is_bf16, long long ld, float* out, int M, int N, float scale, cudaStream_t s);
int pcb_adamw(float* w, const float* g, float* m, float* v, void* w16, long long n, long long n_decay,
              const float* hyper, float b1, float b2, float eps, const float* clip_sumsq, float max_norm,
              cudaStream_t s);
int pcb_f32_to_bf16(const float* x, void* y, long long n, cudaStream_t s);
int pcb_attn_fwd(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H, int HD,
                 float scale, cudaStream_t s);
int pcb_attn_bwd_rope(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                      const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                      int HD, float scale, const float* rope_cs, cudaStream_t s);

int pcb_decode_attn(const void* q, const void* kc, const void* vc, const int* lens, float* pacc, float* pml,
                    void* out, int B, int H, int Hkv, int HD, int cap, int nsplit, float scale, float softcap,
                    cudaStream_t s);
int pcb_wq_gemv(const float* x, const void* w, const float* scale, float* y, int NB, int rows, int cols, int bits,
                cudaStream_t s);
int pcb_softmax_rows(const float* x, float* y, int rows, int n, float scale, cudaStream_t s);
int pcb_softmax_rows_bwd(const float* y, const float* dy, float* dx, int rows, int n, float scale, cudaStream_t s);
int pcb_linear_scan(const float* a, const float* b, float* st, int B, int T, int D, cudaStream_t s);
int pcb_linear_scan_bwd(const float* a, const float* st, const float* ds, float* da, float* db, int B, int T, int D,
                        cudaStream_t s);

int pcb_coll_reduce(const void* const* in_peers, void* out, long long lo, long long hi, int world, int op,
                    float scale, int dtype, int num_sms, cudaStream_t s);
int pcb_coll_reduce_push(const void* const* in_peers, void* const* out_peers, long long lo, long long hi, int world,
                         int op, float scale, int dtype, int num_sms, cudaStream_t s);
int pcb_coll_gather(const void* const* src_peers, void* out, long long chunk, long long src_stride, int world,
                    int dtype, int num_sms, cudaStream_t s);
int pcb_rope_append(const void* qkv, const float* cs_table, const long long* pos, void* qo, void* kc, void* vc, int B,
                    int H, int HD, int cap, cudaStream_t s);
int pcb_swiglu_rows(const void* gu, void* a, int rows, int F, int il16, cudaStream_t s);
long long pcb_checked_violations();
int pcb_attn_bwd_stats(unsigned long long* out);
int pcb_attn_fwd_stats(unsigned long long* out);
int pcb_tp_allreduce_norm(const void* peers, int world, int rows, int D, float* x, const void* gamma, void* y,
                          float eps, void* const* flags, unsigned int* ctr, int rank, int* err, cudaStream_t s);
int pcb_tp_reduce_norm(const void* slots, int world, int rows, int D, const float* resid, float* x_out,
                       int accumulate, const void* gamma, void* y, long long ldy, float* inv, float eps,
                       cudaStream_t s);
int pcb_attn_fwd_tc(const void* qkv, long long ld, void* out, long long ld_o, float* lse, int B, int S, int H,
                    int HD, float scale, int* err, cudaStream_t s);
int pcb_attn_bwd_tc(const void* qkv, long long ld, const void* out, const void* dout, long long ld_o,
                    const float* lse, float* dvec, float* dq_acc, void* dqkv, long long ld_d, int B, int S, int H,
                    int HD, float scale, const float* rope_cs, int* err, cudaStream_t s);
int pcb_annotate(uint8_t* img, int W, int H, const int* boxes, int n, int thickness, const int* segs, int m,
                 const uint8_t* colors, int* owner, cudaStream_t s);
int pcb_alloc(int device, size_t bytes, void* stream, void** out);
int pcb_free(void* ptr);
int pcb_record_stream(void* ptr, void* stream);
void pcb_release_cached(int device);
void pcb_alloc_stats(int device, long long* out6);
void pcb_alloc_reset_peak(int device);
int pcb_stream(int device, int index, int high_priority, int n, void** out);
int pcb_stream_count(int device, int high_priority);

int pcb_peer_alloc(size_t bytes, void** ptr);
int pcb_peer_free(void* ptr);
int pcb_ipc_handle(void* ptr, void* out64);
int pcb_ipc_open(const void* in64, void** ptr);
int pcb_ipc_close(void* ptr);
int pcb_peer_barrier(void* const* peer_flags_dev, unsigned int* ctr, int rank, int world, int* err, cudaStream_t s);
int pcb_dp_reduce_sumsq(const float* grad, const float* staging, long long shard, const long long* tab, int nb,
                        int rank, int world, float* gshard, double* sumsq, int num_sms, cudaStream_t s);
int pcb_dp_norm_push(const double* sumsq, void* const* slot_peers, int rank, int world, cudaStream_t s);
int pcb_dp_adamw_ag(const float* gshard, float* w32, float* m, float* v, void* const* w16_peers, long long shard,
                    const long long* tab, int nb, const float* hyper, float b1, float b2, float eps,
                    const double* norm_slots, float max_norm, int world, int num_sms, cudaStream_t s);
int pcb_memcpy_d2d(void* dst, const void* src, size_t bytes, cudaStream_t s);
int pcb_rs_adamw_ag(void* const* grad_peers, void* const* w16_peers, float* w32, float* m, float* v, long long lo,
                    long long hi, long long n_decay, const float* hyper, float b1, float b2, float eps, int world,
                    int num_sms, cudaStream_t s);
int pcb_pc_allreduce_update(void* const* delta_peers, void* const* w_peers, void* const* w16_peers, long long lo,
                            long long hi, float alpha, float decay, int world, int rank, int num_sms, cudaStream_t s);
int pcb_peer_reduce(void* const* in_peers, void* const* out_peers, long long lo, long long hi, float scale, int world,
                    int num_sms, cudaStream_t s);

int pcb_moe_route(const void* x, long long ldx, const void* router, int M, int D, int E, int k, float* gates,
                  int* topi, cudaStream_t s);
int pcb_moe_dispatch(const int* topi, const float* gates, int M, int k, int E, int cap, int* seg, int* pos, int* src,
                     float* rgate, float* coef, float* loss_acc, float weight, cudaStream_t s);
int pcb_moe_gather(const void* x, long long ldx, const int* src, const int* seg, int E, int D, int cap, void* xs,
                   cudaStream_t s);
int pcb_moe_combine(const float* res, const float* ys, const int* pos, const float* rgate, int M, int k, int D,
                    float* out, cudaStream_t s);
int pcb_moe_combine_bwd(const float* dx, const float* ys, const int* src, const float* rgate, const int* seg, int E,
                        int D, int cap, void* dys, float* dgate, cudaStream_t s);
int pcb_moe_router_bwd(const float* gates, const int* topi, const int* pos, const float* dgate, const float* coef,
                       float weight, const float* dxs, const void* router, int M, int k, int E, int D, float* dlogits,
                       float* dn, cudaStream_t s);
int pcb_moe_router_wgrad(const float* dlogits, const void* x, long long ldx, int M, int E, int D, float* dR,
                         cudaStream_t s);
int pcb_moe_seg_colsum(const void* x, const int* seg, int E, int N, int cap, float* db, cudaStream_t s);

int pcb_skinny_splits(int N, int K, int num_sms);
int pcb_skinny_gemm(const void* x, long long ldx, const void* w, long long ldw, void* y, long long ldy, int y_f32,
                    int M, int N, int K, int splits, int* err, unsigned long long* trace, int swiglu,
                    const SkinnyRope* rope, cudaStream_t stream);

extern "C" void pcb_set_gemm_mode(int mode);

namespace {

std::atomic<long long> g_launches{0};

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc, const char* what, int kernels = 1) {
  g_launches.fetch_add(kernels, std::memory_order_relaxed);
  if (rc == 0) return;
  // Only the numeric CUDA status goes into the message: formatting the runtime's error string here
  // crashed the process on GPU hosts instead of raising.
  const int e = (int)cudaGetLastError();
  PCB_CHECK(false, "pcb kernel '", what, "' failed with code ", rc, " (cuda status ", e, ")");
}

void req(const at::Tensor& t, at::ScalarType dt, const char* name) {
  PCB_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  PCB_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}

// req + contiguous (for kernels that index flat)
void reqc(const at::Tensor& t, at::ScalarType dt, const char* name) {
  req(t, dt, name);
  PCB_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// row stride (elements) of a 2-D view whose inner dimension is contiguous
long long row_stride(const at::Tensor& t, const char* name) {
  PCB_CHECK(t.dim() == 2, name, " must be 2-D");
  PCB_CHECK(t.stride(1) == 1, name, " must have a contiguous inner dimension");
  return t.stride(0);
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

void* ptr_or_null(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// ---------------------------------------------------------------- GEMM
// a: [M,K] (a_mn=0) or [K,M] (a_mn=1);  b: [N,K] (b_mn=0) or [K,N] (b_mn=1).
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int64_t epi,
          const c10::optional<at::Tensor>& c, const c10::optional<at::Tensor>& d,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& bias, double alpha,
          int64_t force_bn, int64_t force_splits, const c10::optional<at::Tensor>& err,
          const c10::optional<at::Tensor>& rope_cs, int64_t rope_S, int64_t rope_hd, int64_t rope_cols,
          const c10::optional<std::vector<int64_t>>& tp) {
  req(a, at::kBFloat16, "a");
  req(b, at::kBFloat16, "b");
  const long long lda = row_stride(a, "a"), ldb = row_stride(b, "b");
  pcb::GemmArgs args{};
  args.M = a_mn ? a.size(1) : a.size(0);
  args.K = a_mn ? a.size(0) : a.size(1);
  args.N = b_mn ? b.size(1) : b.size(0);
  const int kb = b_mn ? b.size(0) : b.size(1);
  PCB_CHECK(kb == args.K, "gemm: K mismatch (", args.K, " vs ", kb, ")");
  args.alpha = static_cast<float>(alpha);
  if (c) { args.C = c->data_ptr(); args.ldc = row_stride(*c, "c"); }
  if (d) { args.D = d->data_ptr(); args.ldd = row_stride(*d, "d"); }
  if (aux) { args.aux = aux->data_ptr(); args.ldaux = row_stride(*aux, "aux"); }
  if (bias) {
    PCB_CHECK(bias->scalar_type() == at::kFloat || bias->scalar_type() == at::kBFloat16, "bias: fp32 or bf16");
    args.bias = bias->data_ptr();
    args.bias_bf16 = bias->scalar_type() == at::kBFloat16 ? 1 : 0;
  }
  if (err) args.err = err->data_ptr<int>();
  if (rope_cs) {
    req(*rope_cs, at::kFloat, "rope_cs");
    PCB_CHECK(epi == pcb::EPI_BF16 && rope_hd % 2 == 0 && rope_S > 0, "gemm: rope needs EPI_BF16, even hd");
    args.rope_cs = rope_cs->data_ptr<float>();
    args.rope_S = (int)rope_S;
    args.rope_hd = (int)rope_hd;
    args.rope_cols = (int)rope_cols;
  }
  if (epi == pcb::EPI_SWIGLU) PCB_CHECK(args.N % 128 == 0, "swiglu gemm needs N % 128 == 0");
  if (epi == pcb::EPI_SWIGLU_BWD) PCB_CHECK(args.N % 64 == 0, "swiglu bwd gemm needs N % 64 == 0");
  if (tp) {
    // tensor-parallel fusion: [ag_peers table, ag_ready counters, ag_rows, ag_rank, ag_world,
    //                          rs_peers table, rs_rows, rs_rank] (device addresses as integers)
    const auto& v = *tp;
    PCB_CHECK(v.size() == 8, "gemm: tp must have 8 entries");
    args.ag_peers = reinterpret_cast<const void* const*>(v[0]);
    args.ag_ready = reinterpret_cast<unsigned int*>(v[1]);
    args.ag_rows = (int)v[2];
    args.ag_rank = (int)v[3];
    args.ag_world = v[0] != 0 ? (int)v[4] : 0;
    args.ag_local = a.data_ptr();
    args.rs_peers = reinterpret_cast<void* const*>(v[5]);
    args.rs_rows = (int)v[6];
    args.rs_rank = (int)v[7];
  }
  if (epi == pcb::EPI_RS_BF16) {
    PCB_CHECK(args.rs_peers != nullptr, "EPI_RS_BF16 needs the tp slot table");
    if (!c) args.ldc = args.N;   // slot buffers are [world * rs_rows, N] row-major
  }
  const at::cuda::CUDAGuard guard(a.device());
  check(pcb_gemm_launch(a.data_ptr(), a_mn, lda, b.data_ptr(), b_mn, ldb, (int)epi, args, (int)force_bn,
                        (int)force_splits, num_sms(), cur_stream()),
        "gemm");
}

// Grouped (mixture-of-experts) GEMM.  mode 1: a [cap, K] sorted activations, b stacks `count` expert
// blocks ([count*N, K], or [count*K, N] with b_mn), bias [count*N]; mode 2 (weight gradients): a [cap, m_per]
// and b [cap, N] read MN-major, c [count*m_per, N] fp32 accumulated.  seg: device int32 [count + 1].
void gemm_grouped(const at::Tensor& a, const at::Tensor& b, bool b_mn, int64_t epi, const at::Tensor& seg,
                  int64_t count, int64_t mode, const c10::optional<at::Tensor>& c, const c10::optional<at::Tensor>& d,
                  const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& bias,
                  const c10::optional<at::Tensor>& err) {
  req(a, at::kBFloat16, "a");
  req(b, at::kBFloat16, "b");
  req(seg, at::kInt, "seg");
  PCB_CHECK(seg.numel() == count + 1, "gemm_grouped: seg must have count + 1 entries");
  PCB_CHECK(mode == 1 || mode == 2, "gemm_grouped: mode 1 (rows) or 2 (weight gradients)");
  const long long lda = row_stride(a, "a"), ldb = row_stride(b, "b");
  pcb::GemmArgs args{};
  int a_mn = 0;
  if (mode == 1) {
    args.M = a.size(0);
    args.K = a.size(1);
    if (b_mn) {
      PCB_CHECK(b.size(0) == count * args.K, "gemm_grouped: b must be [count*K, N]");
      args.N = b.size(1);
    } else {
      PCB_CHECK(b.size(1) == args.K && b.size(0) % count == 0, "gemm_grouped: b must be [count*N, K]");
      args.N = b.size(0) / count;
    }
  } else {
    a_mn = 1;
    PCB_CHECK(b_mn, "gemm_grouped: mode 2 reads b MN-major");
    PCB_CHECK(a.size(0) == b.size(0), "gemm_grouped: a and b must share the sorted rows");
    args.grp_m = a.size(1);
    args.M = count * a.size(1);
    args.K = a.size(0);
    args.N = b.size(1);
  }
  args.alpha = 1.f;
  if (c) { args.C = c->data_ptr(); args.ldc = row_stride(*c, "c"); }
  if (d) { args.D = d->data_ptr(); args.ldd = row_stride(*d, "d"); }
  if (aux) { args.aux = aux->data_ptr(); args.ldaux = row_stride(*aux, "aux"); }
  if (bias) {
    PCB_CHECK(bias->scalar_type() == at::kFloat || bias->scalar_type() == at::kBFloat16, "bias: fp32 or bf16");
    PCB_CHECK(bias->numel() == count * args.N, "gemm_grouped: bias must have count*N entries");
    args.bias = bias->data_ptr();
    args.bias_bf16 = bias->scalar_type() == at::kBFloat16 ? 1 : 0;
  }
  if (err) args.err = err->data_ptr<int>();
  args.grp_seg = seg.data_ptr<int>();
  args.grp_count = (int)count;
  args.grp_mode = (int)mode;
  const at::cuda::CUDAGuard guard(a.device());
  check(pcb_gemm_grouped_launch(a.data_ptr(), a_mn, lda, b.data_ptr(), b_mn ? 1 : 0, ldb, (int)epi, args, num_sms(),
                                cur_stream()),
        "gemm_grouped");
}

// ---------------------------------------------------------------- decode-sized products
// y [M, N] = x [M, K] @ w [K, N] (row-major weight) for M <= 32 on the tcgen05 skinny kernel (K split over
// the CTAs of a cluster, reduced through distributed shared memory; deterministic).
// `trace` (int64, optional) receives 8 globaltimer stamps per CTA: start, weights requested, dependency
// wait over, first tile landed, accumulator read, partials visible, rows stored, end.
void skinny_gemm(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& err,
                 const c10::optional<at::Tensor>& trace, bool swiglu) {
  req(x, at::kBFloat16, "x");
  req(w, at::kBFloat16, "w");
  PCB_CHECK(y.scalar_type() == at::kBFloat16 || y.scalar_type() == at::kFloat, "skinny_gemm: y bf16 or fp32");
  PCB_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(0), "skinny_gemm: x [M, K], w [K, N]");
  PCB_CHECK(x.size(0) <= 32 && y.size(0) == x.size(0) && y.size(1) == (swiglu ? w.size(1) / 2 : w.size(1)),
            "skinny_gemm: M <= 32, y [M, N] ([M, N / 2] with the SwiGLU epilogue)");
  const int M = x.size(0), K = x.size(1), N = w.size(1);
  PCB_CHECK(K % 8 == 0 && N % 8 == 0, "skinny_gemm: K and N must be multiples of 8 (16-byte rows)");
  PCB_CHECK(!swiglu || N % 32 == 0, "skinny_gemm: the SwiGLU epilogue needs N a multiple of 32");
  const at::cuda::CUDAGuard guard(x.device());
  const int splits = pcb_skinny_splits(N, K, num_sms());
  check(pcb_skinny_gemm(x.data_ptr(), row_stride(x, "x"), w.data_ptr(), row_stride(w, "w"), y.data_ptr(),
                        row_stride(y, "y"), y.scalar_type() == at::kFloat ? 1 : 0, M, N, K, splits,
                        err ? err->data_ptr<int>() : nullptr,
                        trace ? reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>()) : nullptr,
                        swiglu ? 1 : 0, nullptr, cur_stream()),
        "skinny_gemm");
}

// One decode token per row: qkv = x @ w on the skinny kernel with the RoPE + KV-append epilogue
// (q rotated into qo [M, H * hd]; k rotated and v appended at row *pos of kc / vc [M, H, cap, hd]).
void skinny_qkv_rope(const at::Tensor& x, const at::Tensor& w, const at::Tensor& cs_table, const at::Tensor& pos,
                     at::Tensor& qo, at::Tensor& kc, at::Tensor& vc) {
  req(x, at::kBFloat16, "x");
  req(w, at::kBFloat16, "w");
  reqc(cs_table, at::kFloat, "cs_table");
  reqc(qo, at::kBFloat16, "qo");
  reqc(kc, at::kBFloat16, "kc");
  reqc(vc, at::kBFloat16, "vc");
  PCB_CHECK(pos.dtype() == at::kLong && pos.is_cuda(), "skinny_qkv_rope: pos must be a cuda int64 scalar tensor");
  PCB_CHECK(kc.dim() == 4 && vc.sizes() == kc.sizes(), "skinny_qkv_rope: caches are [B, H, cap, hd]");
  const int M = x.size(0), K = x.size(1), N = w.size(1);
  const int H = kc.size(1), hd = kc.size(3), cap = kc.size(2);
  PCB_CHECK(x.dim() == 2 && w.dim() == 2 && w.size(0) == K && M <= 32 && kc.size(0) == M && N == 3 * H * hd &&
                qo.numel() == (int64_t)M * H * hd,
            "skinny_qkv_rope: x [M <= 32, K], w [K, 3 H hd], qo [M, H hd], caches [M, H, cap, hd]");
  PCB_CHECK(K % 8 == 0 && N % 8 == 0, "skinny_qkv_rope: K and N must be multiples of 8");
  const at::cuda::CUDAGuard guard(x.device());
  SkinnyRope r{reinterpret_cast<__nv_bfloat16*>(qo.data_ptr()), reinterpret_cast<__nv_bfloat16*>(kc.data_ptr()),
               reinterpret_cast<__nv_bfloat16*>(vc.data_ptr()), cs_table.data_ptr<float>(),
               reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()), H, hd, cap};
  const int splits = pcb_skinny_splits(N, K, num_sms());
  check(pcb_skinny_gemm(x.data_ptr(), row_stride(x, "x"), w.data_ptr(), row_stride(w, "w"), qo.data_ptr(), 0, 0, M,
                        N, K, splits, nullptr, nullptr, 0, &r, cur_stream()),
        "skinny_qkv_rope");
}

// ---------------------------------------------------------------- mixture of experts
void moe_route(const at::Tensor& x, const at::Tensor& router, int64_t k, at::Tensor& gates, at::Tensor& topi) {
  req(x, at::kBFloat16, "x");
  req(router, at::kBFloat16, "router");
  req(gates, at::kFloat, "gates");
  req(topi, at::kInt, "topi");
  const int M = x.size(0), D = x.size(1), E = router.size(0);
  PCB_CHECK(router.size(1) == D && router.is_contiguous(), "moe_route: router must be [E, D] contiguous");
  PCB_CHECK(gates.numel() == (long long)M * E && topi.numel() == (long long)M * k, "moe_route: output sizes");
  check(pcb_moe_route(x.data_ptr(), row_stride(x, "x"), router.data_ptr(), M, D, E, (int)k, gates.data_ptr<float>(),
                      topi.data_ptr<int>(), cur_stream()),
        "moe_route");
}
void moe_dispatch(const at::Tensor& topi, const at::Tensor& gates, int64_t k, at::Tensor& seg, at::Tensor& pos,
                  at::Tensor& src, at::Tensor& rgate, at::Tensor& coef, const c10::optional<at::Tensor>& loss_acc,
                  double weight) {
  req(topi, at::kInt, "topi");
  req(gates, at::kFloat, "gates");
  req(seg, at::kInt, "seg");
  req(pos, at::kInt, "pos");
  req(src, at::kInt, "src");
  req(rgate, at::kFloat, "rgate");
  req(coef, at::kFloat, "coef");
  const int M = gates.size(0), E = gates.size(1);
  PCB_CHECK(seg.numel() == E + 1 && coef.numel() == E && pos.numel() == topi.numel() && topi.numel() == (long long)M * k,
            "moe_dispatch: sizes");
  PCB_CHECK(rgate.numel() == src.numel(), "moe_dispatch: src / rgate sizes");
  check(pcb_moe_dispatch(topi.data_ptr<int>(), gates.data_ptr<float>(), M, (int)k, E, (int)src.numel(),
                         seg.data_ptr<int>(), pos.data_ptr<int>(), src.data_ptr<int>(), rgate.data_ptr<float>(),
                         coef.data_ptr<float>(), loss_acc ? loss_acc->data_ptr<float>() : nullptr, (float)weight,
                         cur_stream()),
        "moe_dispatch");
}
void moe_gather(const at::Tensor& x, const at::Tensor& src, const at::Tensor& seg, at::Tensor& xs) {
  req(x, at::kBFloat16, "x");
  req(xs, at::kBFloat16, "xs");
  req(src, at::kInt, "src");
  req(seg, at::kInt, "seg");
  PCB_CHECK(xs.is_contiguous() && xs.size(1) == x.size(1) && xs.size(0) == src.numel(), "moe_gather: xs shape");
  check(pcb_moe_gather(x.data_ptr(), row_stride(x, "x"), src.data_ptr<int>(), seg.data_ptr<int>(),
                       (int)seg.numel() - 1, x.size(1), (int)src.numel(), xs.data_ptr(), cur_stream()),
        "moe_gather");
}
void moe_combine(const at::Tensor& res, const at::Tensor& ys, const at::Tensor& pos, const at::Tensor& rgate,
                 int64_t k, at::Tensor& out) {
  req(res, at::kFloat, "res");
  req(ys, at::kFloat, "ys");
  req(out, at::kFloat, "out");
  PCB_CHECK(res.is_contiguous() && ys.is_contiguous() && out.is_contiguous(), "moe_combine: contiguous operands");
  check(pcb_moe_combine(res.data_ptr<float>(), ys.data_ptr<float>(), pos.data_ptr<int>(), rgate.data_ptr<float>(),
                        res.size(0), (int)k, res.size(1), out.data_ptr<float>(), cur_stream()),
        "moe_combine");
}
void moe_combine_bwd(const at::Tensor& dx, const at::Tensor& ys, const at::Tensor& src, const at::Tensor& rgate,
                     const at::Tensor& seg, at::Tensor& dys, at::Tensor& dgate) {
  req(dx, at::kFloat, "dx");
  req(ys, at::kFloat, "ys");
  req(dys, at::kBFloat16, "dys");
  req(dgate, at::kFloat, "dgate");
  PCB_CHECK(dx.is_contiguous() && ys.is_contiguous() && dys.is_contiguous(), "moe_combine_bwd: contiguous operands");
  check(pcb_moe_combine_bwd(dx.data_ptr<float>(), ys.data_ptr<float>(), src.data_ptr<int>(), rgate.data_ptr<float>(),
                            seg.data_ptr<int>(), (int)seg.numel() - 1, dx.size(1), (int)src.numel(), dys.data_ptr(),
                            dgate.data_ptr<float>(), cur_stream()),
        "moe_combine_bwd");
}
void moe_router_bwd(const at::Tensor& gates, const at::Tensor& topi, const at::Tensor& pos, const at::Tensor& dgate,
                    const at::Tensor& coef, double weight, const at::Tensor& dxs, const at::Tensor& router, int64_t k,
                    at::Tensor& dlogits, at::Tensor& dn) {
  req(gates, at::kFloat, "gates");
  req(dxs, at::kFloat, "dxs");
  req(router, at::kBFloat16, "router");
  req(dlogits, at::kFloat, "dlogits");
  req(dn, at::kFloat, "dn");
  PCB_CHECK(dxs.is_contiguous() && dn.is_contiguous() && router.is_contiguous(), "moe_router_bwd: contiguous operands");
  const int M = gates.size(0), E = gates.size(1), D = dn.size(1);
  check(pcb_moe_router_bwd(gates.data_ptr<float>(), topi.data_ptr<int>(), pos.data_ptr<int>(), dgate.data_ptr<float>(),
                           coef.data_ptr<float>(), (float)weight, dxs.data_ptr<float>(), router.data_ptr(), M, (int)k, E,
                           D, dlogits.data_ptr<float>(), dn.data_ptr<float>(), cur_stream()),
        "moe_router_bwd");
}
void moe_router_wgrad(const at::Tensor& dlogits, const at::Tensor& x, at::Tensor& dR) {
  req(dlogits, at::kFloat, "dlogits");
  req(x, at::kBFloat16, "x");
  req(dR, at::kFloat, "dR");
  check(pcb_moe_router_wgrad(dlogits.data_ptr<float>(), x.data_ptr(), row_stride(x, "x"), x.size(0), dlogits.size(1),
                             x.size(1), dR.data_ptr<float>(), cur_stream()),
        "moe_router_wgrad");
}
void moe_seg_colsum(const at::Tensor& x, const at::Tensor& seg, at::Tensor& db) {
  req(x, at::kBFloat16, "x");
  req(db, at::kFloat, "db");
  PCB_CHECK(x.is_contiguous(), "moe_seg_colsum: contiguous input");
  const int E = seg.numel() - 1;
  PCB_CHECK(db.numel() == (long long)E * x.size(1), "moe_seg_colsum: db must have E*N entries");
  check(pcb_moe_seg_colsum(x.data_ptr(), seg.data_ptr<int>(), E, x.size(1), x.size(0), db.data_ptr<float>(),
                           cur_stream()),
        "moe_seg_colsum");
}

// PC-specific GEMM entry (epilogues 8..10), scalar knobs passed explicitly.
void gemm_pc(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int64_t epi,
             const c10::optional<at::Tensor>& c, const c10::optional<at::Tensor>& d,
             const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& bias, double alpha, int64_t act,
             double pi, double eta, double actreg, double decay, const c10::optional<at::Tensor>& energy,
             const c10::optional<at::Tensor>& pred_out, const c10::optional<at::Tensor>& pred_bf16,
             const c10::optional<at::Tensor>& err) {
  req(a, at::kBFloat16, "a");
  req(b, at::kBFloat16, "b");
  const long long lda = row_stride(a, "a"), ldb = row_stride(b, "b");
  pcb::GemmArgs args{};
  args.M = a_mn ? a.size(1) : a.size(0);
  args.K = a_mn ? a.size(0) : a.size(1);
  args.N = b_mn ? b.size(1) : b.size(0);
  const int kb = b_mn ? b.size(0) : b.size(1);
  PCB_CHECK(kb == args.K, "gemm_pc: K mismatch");
  args.alpha = static_cast<float>(alpha);
  if (c) { args.C = c->data_ptr(); args.ldc = row_stride(*c, "c"); }
  if (d) { args.D = d->data_ptr(); args.ldd = row_stride(*d, "d"); }
  if (aux) { args.aux = aux->data_ptr(); args.ldaux = row_stride(*aux, "aux"); }
  if (bias) { req(*bias, at::kFloat, "bias"); args.bias = bias->data_ptr(); }
  if (err) args.err = err->data_ptr<int>();
  args.act = (int)act;
  args.pc_pi = (float)pi;
  args.pc_eta = (float)eta;
  args.pc_actreg = (float)actreg;
  args.pc_decay = (float)decay;
  if (energy) args.pc_energy = energy->data_ptr<float>();
  if (pred_out) { args.pc_pred_out = pred_out->data_ptr(); args.ld_pred = row_stride(*pred_out, "pred_out"); }
  if (pred_bf16) {
    args.pc_pred_bf16 = pred_bf16->data_ptr();
    args.ld_pred = row_stride(*pred_bf16, "pred_bf16");
  }
  const at::cuda::CUDAGuard guard(a.device());
  check(pcb_gemm_launch(a.data_ptr(), a_mn, lda, b.data_ptr(), b_mn, ldb, (int)epi, args, 0, 1, num_sms(),
                        cur_stream()),
        "gemm_pc");
}

// ---------------------------------------------------------------- elementwise
void embed_fwd(const at::Tensor& tok, const at::Tensor& W, at::Tensor& x) {
  req(tok, at::kInt, "tok");
  req(W, at::kBFloat16, "W");
  req(x, at::kFloat, "x");
  check(pcb_embed_fwd(tok.data_ptr<int>(), W.data_ptr(), x.data_ptr<float>(), tok.numel(), W.size(1),
                      W.size(0), cur_stream()),
        "embed_fwd");
}
void embed_bwd(const at::Tensor& tok, const at::Tensor& dx, at::Tensor& dW) {
  req(tok, at::kInt, "tok");
  req(dx, at::kFloat, "dx");
  req(dW, at::kFloat, "dW");
  check(pcb_embed_bwd(tok.data_ptr<int>(), dx.data_ptr<float>(), dW.data_ptr<float>(), tok.numel(), dW.size(1),
                      dW.size(0), cur_stream()),
        "embed_bwd");
}
void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& g, at::Tensor& y, const c10::optional<at::Tensor>& inv,
                 double eps) {
  req(x, at::kFloat, "x");
  req(g, at::kBFloat16, "g");
  req(y, at::kBFloat16, "y");
  PCB_CHECK(x.is_contiguous() && y.is_contiguous(), "rmsnorm_fwd: contiguous tensors required");
  const int D = x.size(-1);
  const int M = x.numel() / D;
  check(pcb_rmsnorm_fwd(x.data_ptr<float>(), g.data_ptr(), y.data_ptr(),
                        inv ? inv->data_ptr<float>() : nullptr, M, D, (float)eps, cur_stream()),
        "rmsnorm_fwd");
}
void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& g, const at::Tensor& inv, at::Tensor& dx,
                 const c10::optional<at::Tensor>& dx16, at::Tensor& dg, bool accumulate) {
  req(dy, at::kFloat, "dy");
  req(x, at::kFloat, "x");
  req(g, at::kBFloat16, "g");
  req(dx, at::kFloat, "dx");
  req(dg, at::kFloat, "dg");
  if (dx16) req(*dx16, at::kBFloat16, "dx16");
  const int D = x.size(-1);
  const int M = x.numel() / D;
  check(pcb_rmsnorm_bwd(dy.data_ptr<float>(), x.data_ptr<float>(), g.data_ptr(), inv.data_ptr<float>(),
                        dx.data_ptr<float>(), ptr_or_null(dx16), dg.data_ptr<float>(), M, D, accumulate ? 1 : 0,
                        num_sms(), cur_stream()),
        "rmsnorm_bwd");
}
void rope(at::Tensor& buf, const at::Tensor& cs, int64_t S, int64_t D, int64_t hd, int64_t nparts, double sign) {
  req(buf, at::kBFloat16, "buf");
  req(cs, at::kFloat, "cs");
  const long long ld = row_stride(buf, "buf");
  check(pcb_rope(buf.data_ptr(), ld, cs.data_ptr<float>(), buf.size(0), S, D, hd, nparts, (float)sign, cur_stream()),
        "rope");
}
void cross_entropy(at::Tensor& logits, const at::Tensor& tgt, at::Tensor& loss, double scale, bool write_grad) {
  req(logits, at::kBFloat16, "logits");
  req(tgt, at::kInt, "tgt");
  req(loss, at::kFloat, "loss");
  const long long ld = row_stride(logits, "logits");
  check(pcb_ce(logits.data_ptr(), ld, tgt.data_ptr<int>(), loss.data_ptr<float>(), logits.size(0), logits.size(1),
               (float)scale, write_grad ? 1 : 0, cur_stream()),
        "cross_entropy");
}
void sumsq(const at::Tensor& x, at::Tensor& out, bool square) {
  req(x, at::kFloat, "x");
  req(out, at::kFloat, "out");
  check(pcb_sumsq(x.data_ptr<float>(), x.numel(), out.data_ptr<float>(), square ? 1 : 0, cur_stream()), "sumsq");
}
void colsum(const at::Tensor& x, at::Tensor& out, double scale) {
  PCB_CHECK(x.is_cuda(), "x must be CUDA");
  req(out, at::kFloat, "out");
  const long long ld = row_stride(x, "x");
  const bool bf = x.scalar_type() == at::kBFloat16;
  PCB_CHECK(bf || x.scalar_type() == at::kFloat, "colsum: bf16 or fp32 input");
  check(pcb_colsum(x.data_ptr(), bf ? 1 : 0, ld, out.data_ptr<float>(), x.size(0), x.size(1), (float)scale,
                   cur_stream()),
        "colsum");
}
// hyper: device fp32 [5] = [lr, wd, bias_correction1, bias_correction2, grad_scale]
void adamw(at::Tensor& w, const at::Tensor& g, at::Tensor& m, at::Tensor& v, const c10::optional<at::Tensor>& w16,
           int64_t n_decay, const at::Tensor& hyper, double b1, double b2, double eps,
           const c10::optional<at::Tensor>& clip_sumsq, double max_norm) {
  req(w, at::kFloat, "w");
  req(g, at::kFloat, "g");
  req(m, at::kFloat, "m");
  req(v, at::kFloat, "v");
  if (w16) req(*w16, at::kBFloat16, "w16");
  req(hyper, at::kFloat, "hyper");
  PCB_CHECK(hyper.numel() >= 5, "adamw: hyper needs 5 values");
  check(pcb_adamw(w.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                  ptr_or_null(w16), w.numel(), n_decay, hyper.data_ptr<float>(), (float)b1, (float)b2, (float)eps,
                  clip_sumsq ? clip_sumsq->data_ptr<float>() : nullptr, (float)max_norm, cur_stream()),
        "adamw");
}
void f32_to_bf16(const at::Tensor& x, at::Tensor& y) {
  req(x, at::kFloat, "x");
  req(y, at::kBFloat16, "y");
  PCB_CHECK(x.numel() == y.numel(), "f32_to_bf16: size mismatch");
  check(pcb_f32_to_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), cur_stream()), "f32_to_bf16");
}
void attn_fwd(const at::Tensor& qkv, at::Tensor& out, at::Tensor& lse, int64_t B, int64_t S, int64_t H, int64_t HD,
              double scale) {
  req(qkv, at::kBFloat16, "qkv");
  req(out, at::kBFloat16, "out");
  req(lse, at::kFloat, "lse");
  check(pcb_attn_fwd(qkv.data_ptr(), row_stride(qkv, "qkv"), out.data_ptr(), row_stride(out, "out"),
                     lse.data_ptr<float>(), B, S, H, HD, (float)scale, cur_stream()),
        "attn_fwd");
}
void attn_bwd(const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
              at::Tensor& dvec, at::Tensor& dq_acc, at::Tensor& dqkv, int64_t B, int64_t S, int64_t H, int64_t HD,
              double scale, const c10::optional<at::Tensor>& rope_cs) {
  req(qkv, at::kBFloat16, "qkv");
  req(dout, at::kBFloat16, "dout");
  req(dqkv, at::kBFloat16, "dqkv");
  req(dq_acc, at::kFloat, "dq_acc");
  PCB_CHECK(row_stride(out, "out") == row_stride(dout, "dout"), "attn_bwd: out/dout strides differ");
  if (rope_cs) req(*rope_cs, at::kFloat, "rope_cs");
  check(pcb_attn_bwd_rope(qkv.data_ptr(), row_stride(qkv, "qkv"), out.data_ptr(), dout.data_ptr(),
                          row_stride(dout, "dout"), lse.data_ptr<float>(), dvec.data_ptr<float>(),
                          dq_acc.data_ptr<float>(), dqkv.data_ptr(), row_stride(dqkv, "dqkv"), B, S, H, HD,
                          (float)scale, rope_cs ? rope_cs->data_ptr<float>() : nullptr, cur_stream()),
        "attn_bwd", 3);
}

int64_t launch_count() { return g_launches.load(); }

// ---------------------------------------------------------------- peer memory (CUDA IPC)
// Allocate `bytes` with cudaMalloc (an IPC-exportable allocation base), zeroed, as a uint8 tensor.
at::Tensor peer_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  PCB_CHECK(pcb_peer_alloc((size_t)bytes, &p) == 0, "peer_alloc: cudaMalloc failed");
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  return torch::from_blob(p, {bytes}, [](void* q) { pcb_peer_free(q); }, opts);
}
py::bytes ipc_handle(const at::Tensor& t) {
  char buf[64];
  PCB_CHECK(pcb_ipc_handle(t.data_ptr(), buf) == 0, "ipc_handle: cudaIpcGetMemHandle failed");
  return py::bytes(buf, 64);
}
int64_t ipc_open(py::bytes h) {
  std::string s = h;
  PCB_CHECK(s.size() == 64, "ipc_open: handle must be 64 bytes");
  void* p = nullptr;
  PCB_CHECK(pcb_ipc_open(s.data(), &p) == 0, "ipc_open: cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t p) { pcb_ipc_close(reinterpret_cast<void*>(p)); }

void* const* ptr_table(const at::Tensor& t, int world, const char* name) {
  PCB_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.numel() >= world, name,
              ": device int64 pointer table of size >= world required");
  return reinterpret_cast<void* const*>(t.data_ptr<int64_t>());
}

void peer_barrier(const at::Tensor& flag_ptrs, at::Tensor& ctr, int64_t rank, int64_t world,
                  const c10::optional<at::Tensor>& err) {
  check(pcb_peer_barrier(ptr_table(flag_ptrs, world, "flag_ptrs"), reinterpret_cast<unsigned int*>(ctr.data_ptr()),
                         (int)rank, (int)world, err ? err->data_ptr<int>() : nullptr, cur_stream()),
        "peer_barrier");
}
void rs_adamw_ag(const at::Tensor& grad_ptrs, const at::Tensor& w16_ptrs, at::Tensor& w32, at::Tensor& m, at::Tensor& v,
                 int64_t lo, int64_t hi, int64_t n_decay, const at::Tensor& hyper, double b1, double b2, double eps,
                 int64_t world) {
  req(w32, at::kFloat, "w32");
  PCB_CHECK(w32.numel() >= hi - lo && m.numel() >= hi - lo && v.numel() >= hi - lo, "rs_adamw_ag: state too small");
  check(pcb_rs_adamw_ag(ptr_table(grad_ptrs, world, "grad_ptrs"), ptr_table(w16_ptrs, world, "w16_ptrs"),
                        w32.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), lo, hi, n_decay,
                        hyper.data_ptr<float>(), (float)b1, (float)b2, (float)eps, (int)world, num_sms(), cur_stream()),
        "rs_adamw_ag");
}
void dp_reduce_sumsq(const at::Tensor& grad, const at::Tensor& staging, int64_t shard, const at::Tensor& tab,
                     int64_t rank, int64_t world, at::Tensor& gshard, at::Tensor& sumsq) {
  req(grad, at::kFloat, "grad");
  req(staging, at::kFloat, "staging");
  req(gshard, at::kFloat, "gshard");
  PCB_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kDouble, "dp_reduce_sumsq: sumsq must be a CUDA float64");
  PCB_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.dim() == 2 && tab.size(1) == 4,
            "dp_reduce_sumsq: tab must be a CUDA int64 [buckets, 4] table");
  PCB_CHECK(staging.numel() >= world * shard && gshard.numel() >= shard, "dp_reduce_sumsq: buffers too small");
  check(pcb_dp_reduce_sumsq(grad.data_ptr<float>(), staging.data_ptr<float>(), shard, reinterpret_cast<const long long*>(tab.data_ptr<int64_t>()),
                            (int)tab.size(0), (int)rank, (int)world, gshard.data_ptr<float>(),
                            sumsq.data_ptr<double>(), num_sms(), cur_stream()),
        "dp_reduce_sumsq");
}
void dp_norm_push(const at::Tensor& sumsq, const at::Tensor& slot_ptrs, int64_t rank, int64_t world) {
  PCB_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kDouble, "dp_norm_push: sumsq must be a CUDA float64");
  check(pcb_dp_norm_push(sumsq.data_ptr<double>(), ptr_table(slot_ptrs, world, "slot_ptrs"), (int)rank, (int)world,
                         cur_stream()),
        "dp_norm_push");
}
void dp_adamw_ag(const at::Tensor& gshard, at::Tensor& w32, at::Tensor& m, at::Tensor& v, const at::Tensor& w16_ptrs,
                 int64_t shard, const at::Tensor& tab, const at::Tensor& hyper, double b1, double b2, double eps,
                 const c10::optional<at::Tensor>& norm_slots, double max_norm, int64_t world) {
  req(gshard, at::kFloat, "gshard");
  req(w32, at::kFloat, "w32");
  PCB_CHECK(gshard.numel() >= shard && w32.numel() >= shard && m.numel() >= shard && v.numel() >= shard,
            "dp_adamw_ag: state too small");
  PCB_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.dim() == 2 && tab.size(1) == 4,
            "dp_adamw_ag: tab must be a CUDA int64 [buckets, 4] table");
  if (norm_slots) PCB_CHECK(norm_slots->is_cuda() && norm_slots->scalar_type() == at::kDouble &&
                                norm_slots->numel() >= world, "dp_adamw_ag: norm_slots must be CUDA float64 [world]");
  check(pcb_dp_adamw_ag(gshard.data_ptr<float>(), w32.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                        ptr_table(w16_ptrs, world, "w16_ptrs"), shard, reinterpret_cast<const long long*>(tab.data_ptr<int64_t>()), (int)tab.size(0),
                        hyper.data_ptr<float>(), (float)b1, (float)b2, (float)eps,
                        norm_slots ? norm_slots->data_ptr<double>() : nullptr, (float)max_norm, (int)world, num_sms(),
                        cur_stream()),
        "dp_adamw_ag");
}
void memcpy_d2d(int64_t dst, int64_t src, int64_t bytes) {
  PCB_CHECK(bytes >= 0, "memcpy_d2d: negative size");
  if (bytes == 0) return;
  check(pcb_memcpy_d2d(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), (size_t)bytes, cur_stream()),
        "memcpy_d2d", 0);   // a copy-engine transfer, not a kernel
}
void pc_allreduce_update(const at::Tensor& delta_ptrs, const at::Tensor& w_ptrs, const c10::optional<at::Tensor>& w16_ptrs,
                         int64_t lo, int64_t hi, double alpha, double decay, int64_t world, int64_t rank) {
  check(pcb_pc_allreduce_update(ptr_table(delta_ptrs, world, "delta_ptrs"), ptr_table(w_ptrs, world, "w_ptrs"),
                                w16_ptrs ? ptr_table(*w16_ptrs, world, "w16_ptrs") : nullptr, lo, hi, (float)alpha,
                                (float)decay, (int)world, (int)rank, num_sms(), cur_stream()),
        "pc_allreduce_update");
}
void peer_reduce(const at::Tensor& in_ptrs, const at::Tensor& out_ptrs, int64_t lo, int64_t hi, double scale,
                 int64_t world) {
  check(pcb_peer_reduce(ptr_table(in_ptrs, world, "in_ptrs"), ptr_table(out_ptrs, world, "out_ptrs"), lo, hi,
                        (float)scale, (int)world, num_sms(), cur_stream()),
        "peer_reduce");
}


// ---------------------------------------------------------------- serving / small ops
void decode_attn(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& lens,
                 at::Tensor& pacc, at::Tensor& pml, at::Tensor& out, int64_t nsplit, double scale, double softcap) {
  reqc(q, at::kBFloat16, "q");
  reqc(kc, at::kBFloat16, "k_cache");
  reqc(vc, at::kBFloat16, "v_cache");
  reqc(lens, at::kInt, "lens");
  reqc(pacc, at::kFloat, "pacc");
  reqc(pml, at::kFloat, "pml");
  reqc(out, at::kBFloat16, "out");
  PCB_CHECK(q.dim() == 3 && kc.dim() == 4 && vc.sizes() == kc.sizes(), "decode_attn: q [B,H,hd], caches [B,Hkv,cap,hd]");
  const int64_t B = q.size(0), H = q.size(1), HD = q.size(2), Hkv = kc.size(1), cap = kc.size(2);
  PCB_CHECK(kc.size(0) == B && kc.size(3) == HD && lens.numel() == B, "decode_attn: shape mismatch");
  PCB_CHECK(pacc.numel() >= B * H * nsplit * HD && pml.numel() >= B * H * nsplit * 2, "decode_attn: scratch too small");
  check(pcb_decode_attn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr<int>(), pacc.data_ptr<float>(),
                        pml.data_ptr<float>(), out.data_ptr(), B, H, Hkv, HD, cap, nsplit, (float)scale,
                        (float)softcap, cur_stream()),
        "decode_attn", nsplit > 1 ? 2 : 1);
}
void wq_gemv(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale, at::Tensor& y, int64_t bits) {
  reqc(x, at::kFloat, "x");
  reqc(scale, at::kFloat, "scale");
  reqc(y, at::kFloat, "y");
  PCB_CHECK(w.is_cuda() && w.is_contiguous() && w.element_size() == 1, "wq_gemv: w must be a contiguous byte tensor");
  const int64_t NB = x.size(0), cols = x.size(1), rows = w.size(0);
  PCB_CHECK(w.size(1) == (bits == 8 ? cols : cols / 2) && y.size(0) == NB && y.size(1) == rows, "wq_gemv: shapes");
  check(pcb_wq_gemv(x.data_ptr<float>(), w.data_ptr(), scale.data_ptr<float>(), y.data_ptr<float>(), NB, rows, cols,
                    bits, cur_stream()),
        "wq_gemv");
}
void softmax_rows(const at::Tensor& x, at::Tensor& y, double scale) {
  reqc(x, at::kFloat, "x");
  reqc(y, at::kFloat, "y");
  const int64_t n = x.size(-1), rows = x.numel() / n;
  check(pcb_softmax_rows(x.data_ptr<float>(), y.data_ptr<float>(), rows, n, (float)scale, cur_stream()), "softmax_rows");
}
void softmax_rows_bwd(const at::Tensor& y, const at::Tensor& dy, at::Tensor& dx, double scale) {
  reqc(y, at::kFloat, "y");
  reqc(dy, at::kFloat, "dy");
  reqc(dx, at::kFloat, "dx");
  const int64_t n = y.size(-1), rows = y.numel() / n;
  check(pcb_softmax_rows_bwd(y.data_ptr<float>(), dy.data_ptr<float>(), dx.data_ptr<float>(), rows, n, (float)scale,
                             cur_stream()),
        "softmax_rows_bwd");
}
void linear_scan(const at::Tensor& a, const at::Tensor& b, at::Tensor& s) {
  reqc(a, at::kFloat, "a");
  reqc(b, at::kFloat, "b");
  reqc(s, at::kFloat, "s");
  PCB_CHECK(a.dim() == 3 && a.sizes() == b.sizes() && s.sizes() == a.sizes(), "linear_scan: [B,T,D]");
  check(pcb_linear_scan(a.data_ptr<float>(), b.data_ptr<float>(), s.data_ptr<float>(), a.size(0), a.size(1),
                        a.size(2), cur_stream()),
        "linear_scan");
}
void linear_scan_bwd(const at::Tensor& a, const at::Tensor& s, const at::Tensor& ds, at::Tensor& da, at::Tensor& db) {
  reqc(a, at::kFloat, "a");
  reqc(s, at::kFloat, "s");
  reqc(ds, at::kFloat, "ds");
  reqc(da, at::kFloat, "da");
  reqc(db, at::kFloat, "db");
  check(pcb_linear_scan_bwd(a.data_ptr<float>(), s.data_ptr<float>(), ds.data_ptr<float>(), da.data_ptr<float>(),
                            db.data_ptr<float>(), a.size(0), a.size(1), a.size(2), cur_stream()),
        "linear_scan_bwd");
}


// ---------------------------------------------------------------- collectives over symmetric buffers
int coll_dtype(const at::Tensor& t) {
  if (t.scalar_type() == at::kFloat) return 0;
  PCB_CHECK(t.scalar_type() == at::kBFloat16, "collectives support fp32 and bf16");
  return 1;
}
void coll_reduce(const at::Tensor& in_ptrs, at::Tensor& out, int64_t lo, int64_t hi, int64_t world, int64_t op,
                 double scale) {
  req(in_ptrs, at::kLong, "in_ptrs");
  PCB_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() >= hi - lo, "coll_reduce: out too small");
  check(pcb_coll_reduce(reinterpret_cast<const void* const*>(in_ptrs.data_ptr<int64_t>()), out.data_ptr(), lo, hi,
                        world, op, (float)scale, coll_dtype(out), num_sms(), cur_stream()),
        "coll_reduce");
}
// `like`: a tensor of the payload dtype (the local symmetric buffer)
void coll_reduce_push(const at::Tensor& in_ptrs, const at::Tensor& out_ptrs, const at::Tensor& like, int64_t lo,
                      int64_t hi, int64_t world, int64_t op, double scale) {
  req(in_ptrs, at::kLong, "in_ptrs");
  req(out_ptrs, at::kLong, "out_ptrs");
  PCB_CHECK(in_ptrs.numel() >= world && out_ptrs.numel() >= world, "coll_reduce_push: pointer tables too short");
  check(pcb_coll_reduce_push(reinterpret_cast<const void* const*>(in_ptrs.data_ptr<int64_t>()),
                             reinterpret_cast<void* const*>(out_ptrs.data_ptr<int64_t>()), lo, hi, world, op,
                             (float)scale, coll_dtype(like), num_sms(), cur_stream()),
        "coll_reduce_push");
}
void coll_gather(const at::Tensor& src_ptrs, at::Tensor& out, int64_t chunk, int64_t src_stride, int64_t world) {
  req(src_ptrs, at::kLong, "src_ptrs");
  PCB_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() >= chunk * world, "coll_gather: out too small");
  check(pcb_coll_gather(reinterpret_cast<const void* const*>(src_ptrs.data_ptr<int64_t>()), out.data_ptr(), chunk,
                        src_stride, world, coll_dtype(out), num_sms(), cur_stream()),
        "coll_gather");
}

// ---------------------------------------------------------------- native runtime
at::Tensor dev_alloc(int64_t bytes, int64_t device, int64_t stream) {
  void* p = nullptr;
  PCB_CHECK(pcb_alloc((int)device, (size_t)bytes, reinterpret_cast<void*>(stream), &p) == 0,
              "dev_alloc: out of device memory");
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  return torch::from_blob(p, {bytes}, [](void* q) { pcb_free(q); }, opts);
}
void dev_record_stream(const at::Tensor& t, int64_t stream) {
  PCB_CHECK(pcb_record_stream(t.storage().data_ptr().get(), reinterpret_cast<void*>(stream)) == 0,
              "record_stream: tensor was not allocated by the runtime allocator");
}
std::vector<int64_t> dev_alloc_stats(int64_t device) {
  long long s[6];
  pcb_alloc_stats((int)device, s);
  return std::vector<int64_t>(s, s + 6);
}
int64_t dev_stream(int64_t device, int64_t index, bool high_priority, int64_t n) {
  void* s = nullptr;
  PCB_CHECK(pcb_stream((int)device, (int)index, high_priority ? 1 : 0, (int)n, &s) == 0, "stream creation failed");
  return reinterpret_cast<int64_t>(s);
}


// x_out = (resid or x_out if accumulate or 0) + sum of world bf16 slots; optional RMSNorm into y
void tp_reduce_norm(const at::Tensor& slots, int64_t world, const c10::optional<at::Tensor>& resid, at::Tensor& x_out,
                    bool accumulate, const c10::optional<at::Tensor>& gamma, const c10::optional<at::Tensor>& y,
                    const c10::optional<at::Tensor>& inv, double eps) {
  reqc(slots, at::kBFloat16, "slots");
  reqc(x_out, at::kFloat, "x_out");
  const int64_t rows = x_out.size(0), D = x_out.size(1);
  PCB_CHECK(slots.numel() >= world * rows * D, "tp_reduce_norm: slots too small");
  if (resid) reqc(*resid, at::kFloat, "resid");
  long long ldy = 0;
  if (gamma) {
    PCB_CHECK(y.has_value() && inv.has_value(), "tp_reduce_norm: gamma needs y and inv");
    req(*y, at::kBFloat16, "y");
    ldy = row_stride(*y, "y");
  }
  check(pcb_tp_reduce_norm(slots.data_ptr(), (int)world, (int)rows, (int)D,
                           resid ? resid->data_ptr<float>() : nullptr, x_out.data_ptr<float>(), accumulate ? 1 : 0,
                           gamma ? gamma->data_ptr() : nullptr, y ? y->data_ptr() : nullptr, ldy,
                           inv ? inv->data_ptr<float>() : nullptr, (float)eps, cur_stream()),
        "tp_reduce_norm");
}


// decode helpers: RoPE on one token's q/k + KV-cache append; SwiGLU activation of [rows, 2F] rows
int64_t rope_append(const at::Tensor& qkv, const at::Tensor& cs_table, const at::Tensor& pos, at::Tensor& qo,
                    at::Tensor& kc, at::Tensor& vc) {
  reqc(qkv, at::kBFloat16, "qkv");
  reqc(cs_table, at::kFloat, "cs_table");
  reqc(qo, at::kBFloat16, "qo");
  reqc(kc, at::kBFloat16, "kc");
  reqc(vc, at::kBFloat16, "vc");
  PCB_CHECK(pos.dtype() == at::kLong && pos.is_cuda(), "rope_append: pos must be a cuda int64 scalar tensor");
  PCB_CHECK(kc.dim() == 4, "rope_append: caches are [B, H, cap, HD]");
  return pcb_rope_append(qkv.data_ptr(), cs_table.data_ptr<float>(),
                         reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()), qo.data_ptr(),
                         kc.data_ptr(), vc.data_ptr(), (int)kc.size(0), (int)kc.size(1), (int)kc.size(3),
                         (int)kc.size(2), cur_stream());
}
int64_t swiglu_rows(const at::Tensor& gu, at::Tensor& a, bool interleave16) {
  reqc(gu, at::kBFloat16, "gu");
  reqc(a, at::kBFloat16, "a");
  const int64_t F = a.size(-1);
  PCB_CHECK(gu.size(-1) == 2 * F, "swiglu_rows: gu must be [rows, 2F]");
  return pcb_swiglu_rows(gu.data_ptr(), a.data_ptr(), (int)(a.numel() / F), F, interleave16 ? 1 : 0, cur_stream());
}


// fused all-reduce (peer loads) + residual add + RMSNorm of replicated rows; returns the status
// flags (int64 [world] pointers to [rows, world] int32 flag arrays), ctr (int32 [rows]), rank, err: the
// in-kernel per-row handshake that replaces a device barrier before the reads (all optional together).
int64_t tp_allreduce_norm(const at::Tensor& peers, int64_t world, at::Tensor& x, const at::Tensor& gamma, at::Tensor& y,
                          double eps, const c10::optional<at::Tensor>& flags, const c10::optional<at::Tensor>& ctr,
                          int64_t rank, const c10::optional<at::Tensor>& err) {
  reqc(x, at::kFloat, "x");
  reqc(y, at::kBFloat16, "y");
  req(gamma, at::kBFloat16, "gamma");
  PCB_CHECK(peers.dtype() == at::kLong && peers.numel() >= world, "tp_allreduce_norm: pointer table");
  const int D = x.size(-1);
  const int rows = (int)(x.numel() / D);
  void* const* fl = nullptr;
  unsigned int* c = nullptr;
  if (flags) {
    PCB_CHECK(flags->dtype() == at::kLong && flags->numel() >= world && ctr && ctr->dtype() == at::kInt &&
                  ctr->numel() >= rows && rank >= 0 && rank < world,
              "tp_allreduce_norm: flag pointers [world], epoch counters [rows] int32 and a rank");
    fl = reinterpret_cast<void* const*>(flags->data_ptr<int64_t>());
    c = reinterpret_cast<unsigned int*>(ctr->data_ptr<int>());
  }
  return pcb_tp_allreduce_norm(peers.data_ptr(), (int)world, rows, D, x.data_ptr<float>(), gamma.data_ptr(),
                               y.data_ptr(), (float)eps, fl, c, (int)rank, err ? err->data_ptr<int>() : nullptr,
                               cur_stream());
}


// tcgen05 flash-attention forward (same contract as attn_fwd).  Returns the launcher's status
// (0 ok, -1 unsupported shape, -5 tensor-map encode failure, -(1000 + cudaError) launch failure)
// instead of raising, so the Python caller reports it.
int64_t attn_fwd_tc(const at::Tensor& qkv, at::Tensor& out, at::Tensor& lse, int64_t B, int64_t S, int64_t H,
                    int64_t HD, double scale, const c10::optional<at::Tensor>& err) {
  req(qkv, at::kBFloat16, "qkv");
  req(out, at::kBFloat16, "out");
  reqc(lse, at::kFloat, "lse");
  return pcb_attn_fwd_tc(qkv.data_ptr(), row_stride(qkv, "qkv"), out.data_ptr(), row_stride(out, "out"),
                         lse.data_ptr<float>(), B, S, H, HD, (float)scale, err ? err->data_ptr<int>() : nullptr,
                         cur_stream());
}


// tcgen05 attention backward (same contract as attn_bwd); returns the launcher status like attn_fwd_tc.
int64_t attn_bwd_tc(const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                    at::Tensor& dvec, at::Tensor& dq_acc, at::Tensor& dqkv, int64_t B, int64_t S, int64_t H,
                    int64_t HD, double scale, const c10::optional<at::Tensor>& rope_cs,
                    const c10::optional<at::Tensor>& err) {
  req(qkv, at::kBFloat16, "qkv");
  req(out, at::kBFloat16, "out");
  req(dout, at::kBFloat16, "dout");
  req(dqkv, at::kBFloat16, "dqkv");
  reqc(lse, at::kFloat, "lse");
  reqc(dvec, at::kFloat, "dvec");
  reqc(dq_acc, at::kFloat, "dq_acc");
  return pcb_attn_bwd_tc(qkv.data_ptr(), row_stride(qkv, "qkv"), out.data_ptr(), dout.data_ptr(),
                         row_stride(dout, "dout"), lse.data_ptr<float>(), dvec.data_ptr<float>(),
                         dq_acc.data_ptr<float>(), dqkv.data_ptr(), row_stride(dqkv, "dqkv"), B, S, H, HD,
                         (float)scale, rope_cs ? rope_cs->data_ptr<float>() : nullptr,
                         err ? err->data_ptr<int>() : nullptr, cur_stream());
}


// box outlines + segments rasterised onto a device RGB image (annotation)
void annotate(at::Tensor& img, const at::Tensor& boxes, int64_t thickness, const at::Tensor& segs,
              const at::Tensor& colors, at::Tensor& owner) {
  reqc(img, at::kByte, "img");
  reqc(boxes, at::kInt, "boxes");
  reqc(segs, at::kInt, "segs");
  reqc(colors, at::kByte, "colors");
  reqc(owner, at::kInt, "owner");
  PCB_CHECK(img.dim() == 3 && img.size(2) == 3, "annotate: img must be [H, W, 3]");
  const int64_t H = img.size(0), W = img.size(1);
  const int64_t n = boxes.numel() / 4, m = segs.numel() / 4;
  PCB_CHECK(owner.numel() >= H * W && colors.numel() >= 3 * (n + m), "annotate: scratch or colours too small");
  check(pcb_annotate(img.data_ptr<uint8_t>(), (int)W, (int)H, boxes.data_ptr<int>(), (int)n, (int)thickness,
                     segs.data_ptr<int>(), (int)m, colors.data_ptr<uint8_t>(), owner.data_ptr<int>(), cur_stream()),
        "annotate", 3);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "predicitivecoding_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_pc", &gemm_pc);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("skinny_gemm", &skinny_gemm, py::arg("x"), py::arg("w"), py::arg("y"), py::arg("err") = py::none(),
        py::arg("trace") = py::none(), py::arg("swiglu") = false);
  m.def("skinny_qkv_rope", &skinny_qkv_rope);
  m.def("moe_route", &moe_route);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("moe_router_bwd", &moe_router_bwd);
  m.def("moe_router_wgrad", &moe_router_wgrad);
  m.def("moe_seg_colsum", &moe_seg_colsum);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope", &rope);
  m.def("cross_entropy", &cross_entropy);
  m.def("sumsq", &sumsq);
  m.def("colsum", &colsum);
  m.def("adamw", &adamw);
  m.def("f32_to_bf16", &f32_to_bf16);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_fwd_tc", &attn_fwd_tc);
  m.def("attn_bwd_tc", &attn_bwd_tc);
  m.def("attn_bwd", &attn_bwd);
  m.def("launch_count", &launch_count);
  m.def("_check_status", [](int rc) { check(rc, "status probe", 0); });
  m.def("set_gemm_mode", [](int64_t m) { pcb_set_gemm_mode((int)m); },
        "GEMM kernel choice: -1 env/auto, 0 auto, 1 single-CTA only, 2 CTA pairs when legal");
  m.def("decode_attn", &decode_attn);
  m.def("wq_gemv", &wq_gemv);
  m.def("softmax_rows", &softmax_rows);
  m.def("softmax_rows_bwd", &softmax_rows_bwd);
  m.def("linear_scan", &linear_scan);
  m.def("linear_scan_bwd", &linear_scan_bwd);
  m.def("tp_reduce_norm", &tp_reduce_norm);
  m.def("tp_allreduce_norm", &tp_allreduce_norm, py::arg("peers"), py::arg("world"), py::arg("x"), py::arg("gamma"),
        py::arg("y"), py::arg("eps"), py::arg("flags") = py::none(), py::arg("ctr") = py::none(),
        py::arg("rank") = 0, py::arg("err") = py::none());
  m.def("rope_append", &rope_append);
  m.def("checked_violations", []() { return (int64_t)pcb_checked_violations(); });
  m.def("attn_bwd_stats", []() {
    unsigned long long v[16] = {};
    std::vector<int64_t> out;
    if (pcb_attn_bwd_stats(v) == 0)
      for (int i = 0; i < 16; ++i) out.push_back((int64_t)v[i]);
    return out;
  });
  m.def("attn_fwd_stats", []() {
    unsigned long long v[16] = {};
    std::vector<int64_t> out;
    if (pcb_attn_fwd_stats(v) == 0)
      for (int i = 0; i < 16; ++i) out.push_back((int64_t)v[i]);
    return out;
  });
  m.def("gemm_pair_stats", []() {
    unsigned long long v[12] = {};
    std::vector<int64_t> out;
    if (pcb::pcb_gemm_pair_stats(v) == 0)
      for (int i = 0; i < 12; ++i) out.push_back((int64_t)v[i]);
    return out;
  });
  m.def("swiglu_rows", &swiglu_rows, py::arg("gu"), py::arg("a"), py::arg("interleave16") = false);
  m.def("annotate", &annotate);
  m.def("coll_reduce", &coll_reduce);
  m.def("coll_reduce_push", &coll_reduce_push);
  m.def("coll_gather", &coll_gather);
  m.def("dev_alloc", &dev_alloc);
  m.def("dev_record_stream", &dev_record_stream);
  m.def("dev_release_cached", [](int64_t d) { pcb_release_cached((int)d); });
  m.def("dev_alloc_stats", &dev_alloc_stats);
  m.def("dev_alloc_reset_peak", [](int64_t d) { pcb_alloc_reset_peak((int)d); });
  m.def("dev_stream", &dev_stream);
  m.def("dev_stream_count", [](int64_t d, bool hp) { return pcb_stream_count((int)d, hp ? 1 : 0); });
  m.def("peer_alloc", &peer_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_barrier", &peer_barrier);
  m.def("rs_adamw_ag", &rs_adamw_ag);
  m.def("pc_allreduce_update", &pc_allreduce_update);
  m.def("dp_reduce_sumsq", &dp_reduce_sumsq);
  m.def("dp_norm_push", &dp_norm_push);
  m.def("dp_adamw_ag", &dp_adamw_ag);
  m.def("memcpy_d2d", &memcpy_d2d);
  m.def("peer_reduce", &peer_reduce);
}
