"""Host-side logic of the drop-in boundary that needs no GPU (CPU only)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def test_choose_blocks_respects_psum_banks():
    """tests/test_matmul.py:40-45 of the reference."""
    from nkilab import ops

    for mt in range(1, 9):
        for nt in range(1, 17):
            bm, bn = ops.choose_blocks(mt, nt)
            assert bm * bn <= 8 and mt % bm == 0 and nt % bn == 0
    assert ops.choose_blocks(4, 4) in {(2, 4), (4, 2)}


def test_choose_blocks_matches_reference_table():
    from nkilab import ops

    with open(os.path.join(GOLDEN, "golden_blocks.json")) as f:
        table = json.load(f)
    for key, want in table.items():
        m, n = map(int, key.split(","))
        assert list(ops.choose_blocks(m, n)) == want


def test_blocked_rejects_psum_overflow():
    """tests/test_matmul.py:33-37 of the reference: BM=BN=3 fails with 'PSUM'."""
    from nkilab.kernels import matmul as mm

    lhsT = np.zeros((128, 384), np.float32)
    rhs = np.zeros((128, 1536), np.float32)
    with pytest.raises(Exception, match="PSUM"):
        mm.matmul_blocked(lhsT, rhs, BM=3, BN=3)


def test_kernel_level_shape_asserts():
    from nkilab.kernels import attention as at
    from nkilab.kernels import matmul as mm

    with pytest.raises(AssertionError):
        mm.matmul_naive(np.zeros((100, 128), np.float32), np.zeros((100, 512), np.float32))
    with pytest.raises(AssertionError):
        at.flash_attention(np.zeros((1, 64, 100), np.float32), np.zeros((1, 64, 100), np.float32),
                           np.zeros((1, 100, 64), np.float32), 0.125)


def test_ops_argument_errors_before_any_device_work():
    from nkilab import ops

    with pytest.raises(AssertionError):
        ops.matmul(np.zeros((4, 5), np.float32), np.zeros((6, 3), np.float32))
    with pytest.raises(KeyError):
        ops.attention(np.zeros((1, 4, 8), np.float32), np.zeros((1, 4, 8), np.float32),
                      np.zeros((1, 4, 8), np.float32), variant="nope")
    with pytest.raises(AssertionError):
        ops.attention(np.zeros((1, 4, 256), np.float32), np.zeros((1, 4, 256), np.float32),
                      np.zeros((1, 4, 256), np.float32))


def test_attention_variants_keys_match_reference():
    from nkilab import ops

    assert list(ops.ATTENTION_VARIANTS) == ["naive", "flash", "flash_kv_resident", "flash_balanced",
                                            "flash_pipelined"]


def test_ops_refuse_cpu_execution():
    """No CPU fallback: the custom ops raise on CPU tensors."""
    import torch

    from nkilab import _torch_ops  # noqa: F401

    x = torch.zeros(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.nkilab.softmax(x, True)


def test_block_weights_follow_reference_seeding():
    import torch

    from nkilab.model import BlockConfig, DecoderBlock

    torch.manual_seed(0)
    b = DecoderBlock(BlockConfig())
    names = [n for n, _ in b.named_parameters()]
    assert names == ["norm1.weight", "norm2.weight", "wqkv.weight", "wo.weight", "wg.weight", "wu.weight", "wd.weight"]
    w1 = b.norm1.weight.detach()
    assert float(w1.min()) >= 0.5 and float(w1.max()) <= 1.5


def test_eager_attention_workspace_grows_per_stream():
    """Eager calls share one workspace per (device, stream), reused while large enough and
    replaced when a larger shape needs more (graphs never hold the eager workspace: a
    call under stream capture takes its own from the graph's memory pool)."""
    import torch

    from nkilab import _torch_ops as T

    dev, stream = torch.device("cpu"), -12345  # a key no real stream uses
    small = T._attention_workspace(dev, stream, 256)
    assert T._attention_workspace(dev, stream, 128) is small  # big enough: reused
    big = T._attention_workspace(dev, stream, 1024)
    assert big is not small and big.numel() >= 1024
    assert T._attention_workspace(dev, stream, 512) is big
    assert T._attention_workspace(dev, -54321, 64) is not big  # another stream: its own
    T._attention_ws.pop((dev.index, stream))
    T._attention_ws.pop((dev.index, -54321))
