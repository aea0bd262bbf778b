"""CLI entry points: translation tool, demo menu, mixed-precision benchmark (CPU)."""
import os

import pytest

from predicitivecoding_b200.cli import demos, mixed_precision_bench, translate


def test_arg_map():
    a = translate.arg_map(["--corpus", "x.tsv", "--dim", "64", "--verbose"])
    assert a == {"corpus": "x.tsv", "dim": "64", "verbose": "true"}


def test_gradcheck_passes():
    assert translate.gradcheck()


def test_train_then_translate(tmp_path, capsys):
    tsv = tmp_path / "pairs.tsv"
    rows = [("it", "cat", "gatto"), ("it", "dog", "cane"), ("it", "house", "casa"), ("it", "sun", "sole")] * 8
    tsv.write_text("\n".join("\t".join(r) for r in rows) + "\n")
    out = tmp_path / "model"
    rc = translate.main(["train", "--corpus", str(tsv), "--out", str(out), "--dim", "32", "--blocks", "1",
                         "--heads", "2", "--maxseq", "32", "--merges", "40", "--epochs", "30", "--batch", "8",
                         "--lr", "0.01"])
    assert rc == 0 and os.path.isdir(out)
    assert translate.main(["translate", "--model", str(out), "--text", "dog", "--to", "it"]) == 0
    assert "cane" in capsys.readouterr().out


def test_translate_usage_errors():
    assert translate.main(["train"]) == 2
    assert translate.main(["translate"]) == 2
    assert translate.main(["nope"]) == 2
    assert translate.main([]) == 0


@pytest.mark.parametrize("key", ["1", "2", "3", "4", "5", "6", "7", "8", "9", "10", "11", "12"])
def test_demos_run(key):
    assert isinstance(demos.DEMOS[key][1](), str)


def test_mixed_precision_rows():
    rows = mixed_precision_bench.run()
    names = [r[0] for r in rows]
    assert names.count("MatVec") == 2 and "GEMM" in names
    assert all(r[2] > 0 and r[3] > 0 for r in rows)


def test_demo_menu_covers_the_reference_thirteen():
    assert sorted(demos.DEMOS, key=int) == [str(i) for i in range(1, 14)]
