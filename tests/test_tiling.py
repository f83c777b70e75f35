"""The GEMM tiling rules the step applies (CPU: pure functions of the shapes)."""
from r97training_b200 import ops


def test_grad_tiling_rule():
    """The adapter-gradient tiling at the config-5 shapes: the split counts measured best on B200."""
    assert ops.grad_tiling(12288, 64) == (64, 3)
    assert ops.grad_tiling(4096, 64) == (64, 4)
    assert ops.grad_tiling(8192, 64) == (64, 2)
    assert ops.grad_tiling(4096, 192) == (128, 2)
    assert ops.grad_tiling(64, 64) == (64, 8)
    assert ops.grad_tiling(64, 64, K=2048) == (64, 2)   # K / s >= 1024


def test_skinny_tiling_rule():
    """The narrow products' tiling at the config-5 shapes (M = 8192 tokens): bn 64 up to 64 columns, else
    128; a split in two when the tiles would fill under 100 SMs and the split pays (64 columns, or K >= 8192)."""
    assert ops.skinny_tiling(8192, 64, 4096) == (64, 2)
    assert ops.skinny_tiling(8192, 128, 4096) == (128, 1)
    assert ops.skinny_tiling(8192, 128, 24576) == (128, 2)
    assert ops.skinny_tiling(8192, 192, 10240) == (128, 1)
