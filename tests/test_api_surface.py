"""CPU checks of the drop-in Python surface (no GPU needed).

The reference package exports 21 names plus ``__version__``
(batch_invariant_ops/__init__.py:1-48 of yiannisha/robotics-batch-invariant-ops);
user code written against it must find the same names here.  vLLM's
attention-backend hook reads a constant (16, 16) block size
(batch_invariant_ops.py:1715-1719).  CPU tensors never take a silent CPU
path: the operators raise the reference's exception types.
"""

from __future__ import annotations

import pytest
import torch

import batch_invariant_ops as bio

REFERENCE_NAMES = (
    "set_batch_invariant_mode", "is_batch_invariant_mode_enabled",
    "disable_batch_invariant_mode", "enable_batch_invariant_mode", "matmul_persistent",
    "linear_batch_invariant", "bmm_persistent", "conv1d_batch_invariant",
    "conv2d_batch_invariant", "conv3d_batch_invariant", "conv_transpose2d_batch_invariant",
    "conv_transpose3d_batch_invariant", "scaled_dot_product_attention_batch_invariant",
    "varlen_scaled_dot_product_attention_batch_invariant", "linalg_vector_norm_batch_invariant",
    "softmax", "log_softmax", "mean_dim", "get_batch_invariant_attention_block_size",
    "AttentionBlockSize", "deterministic_token_choice_moe",
)


def test_reference_names_and_version_are_exported():
    for name in REFERENCE_NAMES:
        assert hasattr(bio, name), name
        assert name in bio.__all__, name
    assert bio.__version__ == "0.2.0"


def test_attention_block_size_constant_for_vllm_hook():
    size = bio.get_batch_invariant_attention_block_size()
    assert size == bio.AttentionBlockSize(block_m=16, block_n=16)
    assert size == (16, 16)
    assert bio.AttentionBlockSize._fields == ("block_m", "block_n")
    assert size.block_m == 16 and size.block_n == 16


def test_mode_context_is_reentrant_and_exception_safe_flag():
    # the flag logic alone (registration needs the accelerator key, which is
    # exercised on the GPU); disabled state is restored after an exception
    assert not bio.is_batch_invariant_mode_enabled()
    with pytest.raises(RuntimeError):
        with bio.set_batch_invariant_mode(False):
            raise RuntimeError("boom")
    assert not bio.is_batch_invariant_mode_enabled()


@pytest.mark.parametrize(
    "call",
    [
        lambda: bio.matmul_persistent(torch.randn(4, 8), torch.randn(8, 3)),
        lambda: bio.bmm_persistent(torch.randn(2, 4, 8), torch.randn(2, 8, 3)),
        lambda: bio.linear_batch_invariant(torch.randn(4, 8), torch.randn(3, 8)),
        lambda: bio.log_softmax(torch.randn(4, 8)),
        lambda: bio.mean_dim(torch.randn(4, 8), -1),
        lambda: bio.linalg_vector_norm_batch_invariant(torch.randn(4, 8), dim=1),
        lambda: bio.conv2d_batch_invariant(torch.randn(1, 3, 8, 8), torch.randn(4, 3, 3, 3), None,
                                           (1, 1), (0, 0), (1, 1), False, (0, 0), 1),
    ],
)
def test_cpu_tensors_raise_assertion_instead_of_running_on_cpu(call):
    with pytest.raises(AssertionError):
        call()


def test_cpu_tensors_raise_for_value_error_family():
    # softmax / SDPA validate with ValueError first (reference :1124-1127,
    # :1166-1185); CPU tensors then still refuse to run
    with pytest.raises((AssertionError, ValueError)):
        bio.softmax(torch.randn(4, 8))
    q = torch.randn(1, 2, 4, 8)
    with pytest.raises((AssertionError, ValueError)):
        bio.scaled_dot_product_attention_batch_invariant(q, q, q)
    with pytest.raises(ValueError):
        bio.scaled_dot_product_attention_batch_invariant(q, q, q, dropout_p=0.1)
