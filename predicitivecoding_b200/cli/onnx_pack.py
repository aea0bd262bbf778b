"""Convert an ``.onnx`` model to the in-house PCNX format.

Reference: tools/OnnxPack/Program.cs (``OnnxPack <input.onnx> [output.pcnx] [--no-optimize]``;
optimisation folds constants, drops Identity nodes and dead code; the output is re-loaded to
prove it parses and the node / initializer counts and sizes are printed).
"""
from __future__ import annotations

import os
import sys
from typing import List

from ..systems.onnx import OnnxModel, optimize_graph, write_pcnx


def main(argv: List[str] = None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    optimize = "--no-optimize" not in argv
    unknown = [a for a in argv if a.startswith("--") and a != "--no-optimize"]
    paths = [a for a in argv if not a.startswith("--")]
    if unknown:
        print(f"Unknown option(s): {', '.join(unknown)}. Did you mean --no-optimize?", file=sys.stderr)
        return 1
    if not 1 <= len(paths) <= 2:
        print("Convert a .onnx model to the in-house PCNX format.\n\n"
              "  Usage: python -m predicitivecoding_b200.cli.onnx_pack <input.onnx> [output.pcnx] [--no-optimize]")
        return 1
    src = paths[0]
    dst = paths[1] if len(paths) == 2 else os.path.splitext(src)[0] + ".pcnx"
    if not os.path.isfile(src):
        print(f"Input not found: {src}", file=sys.stderr)
        return 1
    if os.path.abspath(src) == os.path.abspath(dst):
        print("Output path equals the input path; pick a different output file.", file=sys.stderr)
        return 1
    model = OnnxModel.load(src)
    g = optimize_graph(model.graph) if optimize else model.graph
    write_pcnx(dst, g)
    back = OnnxModel.load(dst)
    print(f"  {src}  ->  {dst}")
    print(f"  nodes        : {len(model.graph.nodes)} -> {len(back.graph.nodes)}" + ("" if optimize else "  (no optimization)"))
    print(f"  initializers : {len(model.graph.initializers)} -> {len(back.graph.initializers)}")
    print(f"  file size    : {os.path.getsize(src) / 2**20:.1f} MB -> {os.path.getsize(dst) / 2**20:.1f} MB")
    print(f"  inputs       : {', '.join(back.input_names)}")
    print(f"  outputs      : {', '.join(back.output_names)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
