"""Runtime kernel compilation (NVRTC, no GPU needed) and the evaluation bundle."""
import pytest
import torch

from predicitivecoding_b200.runtime.kernel import I64, KernelCompileError, RuntimeKernel, compile_cubin

SAXPY = r'''
extern "C" __global__ void saxpy(float a, const float* x, float* y, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = a * x[i] + y[i];
}'''


def test_nvrtc_compiles_for_sm100a_and_reports_errors():
    assert len(compile_cubin(SAXPY)) > 0
    with pytest.raises(KernelCompileError) as e:
        compile_cubin('extern "C" __global__ void k() { not_declared(); }')
    assert "not_declared" in str(e.value)


def test_argument_marshalling():
    holders, ptrs = RuntimeKernel._marshal([torch.zeros(4), 3, 2.5, I64(1 << 40)])
    assert len(holders) == len(ptrs) == 4
    assert holders[1].value == 3 and abs(holders[2].value - 2.5) < 1e-7 and holders[3].value == 1 << 40
    with pytest.raises(TypeError):
        RuntimeKernel._marshal(["no"])


def test_pro_eval_bundle_and_corpus():
    from predicitivecoding_b200.llm.eval import eval_corpus, pro_eval
    from predicitivecoding_b200.llm.facade import PredictiveLlm
    llm = PredictiveLlm.create_pc(dim=32, blocks=1, heads=2, ff_dim=64, max_seq=64)
    text = eval_corpus()
    assert text.count("\n") >= 9
    rep = pro_eval(llm, text, {"corpus": text, "digits": "0123456789 " * 10}, serve_tokens=8)
    assert rep.bits_per_byte.bits_per_byte > 0
    assert set(rep.per_domain_perplexity) == {"corpus", "digits"}
    assert 0.0 <= rep.probes.echo <= 1.0 and 0.0 <= rep.probes.induction <= 1.0
    assert rep.serve_tokens_per_second > 0
