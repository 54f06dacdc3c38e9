"""The torch.library override surface (reference batch_invariant_ops.py:1654-1712):
inside ``set_batch_invariant_mode`` stock torch calls reach the sm_100a
kernels and become batch invariant (reference test_batch_invariance.py:407-792)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from batch_invariant_ops import is_batch_invariant_mode_enabled, set_batch_invariant_mode
from conftest import DTYPES, TOLERANCES, assert_first_sample_equal

pytestmark = pytest.mark.gpu


def test_mode_overrides_matmul_and_convolution_family():
    gen = torch.Generator(device="cuda").manual_seed(7000)

    def rn(*s):
        return torch.randn(*s, device="cuda", generator=gen)

    query, key = rn(5, 19, 23), rn(5, 23, 17)
    image, weight = rn(5, 3, 28, 28), rn(8, 3, 14, 14)
    signal, signal_weight = rn(5, 8, 19), rn(8, 1, 4)
    video, video_weight = rn(5, 3, 2, 16, 16), rn(8, 3, 2, 16, 16)
    latent, transpose_weight = rn(5, 8, 2, 3, 3), rn(8, 6, 4, 1, 1)
    image_latent, image_transpose_weight = rn(5, 8, 3, 3), rn(8, 6, 4, 4)
    linear_input, linear_weight, linear_bias = rn(5, 37, 257), rn(91, 257), rn(91)
    with set_batch_invariant_mode():
        assert_first_sample_equal(query[:1] @ key[:1], query @ key)
        assert_first_sample_equal(F.linear(linear_input[:1], linear_weight, linear_bias),
                                  F.linear(linear_input, linear_weight, linear_bias))
        assert_first_sample_equal(F.conv1d(signal[:1], signal_weight, padding=3, groups=8),
                                  F.conv1d(signal, signal_weight, padding=3, groups=8))
        assert_first_sample_equal(F.conv2d(image[:1], weight, stride=14), F.conv2d(image, weight, stride=14))
        assert_first_sample_equal(F.conv3d(video[:1], video_weight, stride=(2, 16, 16)),
                                  F.conv3d(video, video_weight, stride=(2, 16, 16)))
        assert_first_sample_equal(F.conv_transpose3d(latent[:1], transpose_weight, stride=(4, 1, 1)),
                                  F.conv_transpose3d(latent, transpose_weight, stride=(4, 1, 1)))
        assert_first_sample_equal(F.conv_transpose2d(image_latent[:1], image_transpose_weight, stride=4),
                                  F.conv_transpose2d(image_latent, image_transpose_weight, stride=4))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch_size", (2, 5, 17))
@pytest.mark.parametrize("dim", (-1, 1))
def test_mode_overrides_torch_softmax(dtype, batch_size, dim):
    gen = torch.Generator(device="cuda").manual_seed(7025 + batch_size)
    x = torch.randn(batch_size, 7, 145, device="cuda", generator=gen).to(dtype)
    with set_batch_invariant_mode():
        assert_first_sample_equal(torch.softmax(x[:1], dim=dim), torch.softmax(x, dim=dim))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", (-1, 1))
def test_mode_softmax_and_log_softmax_match_torch(dtype, dim):
    gen = torch.Generator(device="cuda").manual_seed(7040 + dim)
    x = torch.randn(3, 7, 145, device="cuda", generator=gen).to(dtype)
    expected = torch.softmax(x, dim=dim), torch.log_softmax(x, dim=dim)
    with set_batch_invariant_mode():
        actual = torch.softmax(x, dim=dim), torch.log_softmax(x, dim=dim)
    torch.testing.assert_close(actual[0], expected[0], **TOLERANCES[dtype])
    torch.testing.assert_close(actual[1], expected[1], **TOLERANCES[dtype])


@pytest.mark.parametrize("composition", ("duplicate", "unrelated"))
def test_rms_normalization_is_batch_invariant(composition):
    gen = torch.Generator(device="cuda").manual_seed(7075)
    target = torch.randn(1, 1024, 4, 33, 40, device="cuda", generator=gen).to(torch.bfloat16)
    if composition == "duplicate":
        inputs = target.repeat(2, 1, 1, 1, 1)
    else:
        companion = torch.randn(1, 1024, 4, 33, 40, device="cuda", generator=gen).to(torch.bfloat16)
        inputs = torch.cat((target, companion))
    with set_batch_invariant_mode():
        alone = F.normalize(target, dim=1)
        batched = F.normalize(inputs, dim=1)
    assert_first_sample_equal(alone, batched)


def test_mode_overrides_scaled_dot_product_attention():
    gen = torch.Generator(device="cuda").manual_seed(7300)
    q = torch.randn(3, 16, 256, 72, device="cuda", generator=gen).to(torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    with set_batch_invariant_mode():
        alone = F.scaled_dot_product_attention(q[:1], k[:1], v[:1])
        batched = F.scaled_dot_product_attention(q, k, v)
    assert_first_sample_equal(alone, batched)


def test_mode_overrides_mean_and_addmm():
    gen = torch.Generator(device="cuda").manual_seed(7310)
    x = torch.randn(9, 300, device="cuda", generator=gen).to(torch.bfloat16)
    w = torch.randn(300, 70, device="cuda", generator=gen).to(torch.bfloat16)
    b = torch.randn(70, device="cuda", generator=gen).to(torch.bfloat16)
    with set_batch_invariant_mode():
        assert_first_sample_equal(x[:1].mean(dim=-1), x.mean(dim=-1))
        assert_first_sample_equal(torch.addmm(b, x[:1], w), torch.addmm(b, x, w))
        m2 = x.reshape(9, 3, 100).mean(dim=(1, 2))
    torch.testing.assert_close(m2, x.reshape(9, 3, 100).mean(dim=(1, 2)), **TOLERANCES[torch.bfloat16])


def test_mode_context_is_exception_safe_and_reentrant():
    assert not is_batch_invariant_mode_enabled()
    with pytest.raises(RuntimeError, match="sentinel"):
        with set_batch_invariant_mode():
            assert is_batch_invariant_mode_enabled()
            with set_batch_invariant_mode():
                assert is_batch_invariant_mode_enabled()
            assert is_batch_invariant_mode_enabled()
            raise RuntimeError("sentinel")
    assert not is_batch_invariant_mode_enabled()


def test_mode_addmm_beta_alpha():
    gen = torch.Generator(device="cuda").manual_seed(7311)
    x = torch.randn(9, 300, device="cuda", generator=gen).to(torch.bfloat16)
    w = torch.randn(300, 70, device="cuda", generator=gen).to(torch.bfloat16)
    b = torch.randn(70, device="cuda", generator=gen).to(torch.bfloat16)
    ref = torch.addmm(b.float(), x.float(), w.float(), beta=0.5, alpha=2.0)
    with set_batch_invariant_mode():
        full = torch.addmm(b, x, w, beta=0.5, alpha=2.0)
        assert_first_sample_equal(torch.addmm(b, x[:1], w, beta=0.5, alpha=2.0), full)
        no_bias = torch.addmm(b, x, w, beta=0, alpha=1.5)
    torch.testing.assert_close(full.float(), ref, **TOLERANCES[torch.bfloat16])
    torch.testing.assert_close(no_bias.float(), 1.5 * (x.float() @ w.float()),
                               **TOLERANCES[torch.bfloat16])


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
@pytest.mark.parametrize("op", (torch.ops.aten._softmax, torch.ops.aten._log_softmax))
def test_mode_softmax_half_to_float(dtype, op):
    gen = torch.Generator(device="cuda").manual_seed(7312)
    x = (torch.randn(6, 5, 1000, device="cuda", generator=gen) * 3).to(dtype)
    ref = op(x.float(), -1, False)
    with set_batch_invariant_mode():
        full = op(x, -1, True)
        alone = op(x[:1], -1, True)
    assert full.dtype == torch.float32
    assert_first_sample_equal(alone, full)
    torch.testing.assert_close(full, ref, rtol=1e-5, atol=1e-6)
