"""The profiling targets (`python -m tosa_b200.profile_layer ...`) run on small layers."""

import pytest

from tosa_b200 import profile_layer


@pytest.mark.gpu
@pytest.mark.parametrize("argv", [["conv", "2", "8", "64", "64", "3", "--runs", "3"],
                                  ["depthwise", "2", "8", "32", "3", "2", "--runs", "3"],
                                  ["residual", "2", "8", "64", "--runs", "3"],
                                  ["matmul_t", "2", "64", "128", "96", "1", "--runs", "3"]])
def test_profile_layer_runs(argv, capsys):
    assert profile_layer.main(argv) == 0
    assert " us" in capsys.readouterr().out
