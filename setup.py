"""Build the sm_100a kernels of predicitivecoding_b200 in-tree.

    python setup.py build_ext --inplace

produces predicitivecoding_b200/_C*.so next to the Python sources.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("predicitivecoding_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def _shared_libstdcxx() -> list:
    """Link the extension against the C++ runtime this interpreter has loaded (a shared libstdc++).

    When the compiler driver finds only a static libstdc++ it embeds a second copy of the runtime in the
    extension; that copy's locale is never initialised inside the Python process, and formatting a
    number into an error message then crashes instead of raising.
    """
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.split()[-1]
                if "/libstdc++.so" in path and os.path.exists(path):
                    return [path]
    except OSError:
        pass
    return []


if os.environ.get("PCB_CHECKED") == "1":   # debug build: bounds-violation counters in the kernels
    NVCC_FLAGS.append("-DPCB_CHECKED")
if os.environ.get("PCB_GEMM_STATS") == "1":   # profiling build: cycle counters in the pair GEMM roles
    NVCC_FLAGS.append("-DPCB_GEMM_STATS")
if os.environ.get("PCB_ATTN_STATS") == "1":   # profiling build: cycle counters in the attention backward roles
    NVCC_FLAGS.append("-DPCB_ATTN_STATS")

setup(
    name="predicitivecoding_b200",
    version="0.1.0",
    packages=["predicitivecoding_b200"],
    ext_modules=[
        CUDAExtension(
            name="predicitivecoding_b200._C",
            sources=[
                os.path.join(CSRC, "bindings.cpp"),
                os.path.join(CSRC, "gemm_tcgen05.cu"),
                os.path.join(CSRC, "gemm2_tcgen05.cu"),
                os.path.join(CSRC, "ops_llm.cu"),
                os.path.join(CSRC, "attention.cu"),
                os.path.join(CSRC, "attention_tc.cu"),
                os.path.join(CSRC, "attention_bwd_tc.cu"),
                os.path.join(CSRC, "attention_bwd_tc128.cu"),
                os.path.join(CSRC, "peer.cu"),
                os.path.join(CSRC, "decode.cu"),
                os.path.join(CSRC, "collectives.cu"),
                os.path.join(CSRC, "tp.cu"),
                os.path.join(CSRC, "vision.cu"),
                os.path.join(CSRC, "moe.cu"),
                os.path.join(CSRC, "skinny.cu"),
                os.path.join(CSRC, "runtime.cpp"),
            ],
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            extra_link_args=_shared_libstdcxx(),
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
