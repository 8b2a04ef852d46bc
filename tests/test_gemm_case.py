"""The K3 case runner (zest_b200.gemm_case) on the host: its shapes are the
configs' layer launches, every K a whole number of 64-column k-blocks, and
an unknown shape name is refused before any GPU work."""
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)), "ggml-xdna_b200"))
from zest_b200 import gemm_case  # noqa: E402


def test_shapes_are_the_configs_launches():
    assert gemm_case.SHAPES["C1"] == (1024, [9728], 2560)
    assert gemm_case.SHAPES["C2 down"] == (8192, [2560], 9728)
    for name, (M, Ns, K) in gemm_case.SHAPES.items():
        assert K % 64 == 0 and M > 0 and 1 <= len(Ns) <= 4, name


def test_unknown_shape_refused():
    with pytest.raises(SystemExit):
        gemm_case.main(["no such shape"])


def test_plan_lines_without_gpu(capsys):
    gemm_case.main(["--plan", "C1", "C3 o"])
    import json
    plans = [json.loads(x) for x in capsys.readouterr().out.splitlines()]
    assert [p["shape"] for p in plans] == ["C1", "C3 o"]
    assert plans[0]["stream_k"] == 0 and plans[1]["stream_k"] == 1
