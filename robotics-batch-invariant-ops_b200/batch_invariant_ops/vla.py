"""Random-init pi0-style vision-language-action step.

A SigLIP-like vision tower (patch-14 conv, pre-LN transformer), a Gemma-like
prefix language model (grouped-query attention, RMSNorm, GeGLU) over
[image tokens, text tokens], and an action expert that attends jointly to the
prefix keys/values of its layer and to the action tokens, integrated with a
fixed number of flow-matching (Euler) steps over an action chunk.  Written
with stock torch.nn.functional calls only, so that under
``set_batch_invariant_mode`` every GEMM, convolution, attention, softmax and
mean runs on this library's kernels; when the mode is on, the GeGLU input
projections call the library's fused gated GEMM
(``gated_linear_batch_invariant``) and the residual adds after the output
projections ride in the GEMM's epilogue
(``linear_residual_batch_invariant``), with the stock ops' rounding steps.  The weights are random (no checkpoint) and the inputs synthetic.

``VLAConfig.full()`` is the BASELINE size (So400m-like 27 x 1152 vision
tower, Gemma-2B-like 18 x 2048 prefix LM with 8 query / 1 KV heads of 256,
300M-class action expert, 10 steps over a 50 x 32 chunk); ``VLAConfig.tiny()``
keeps every structural feature at test size.  ``VLAAdapter`` plugs the model
into ``model_invariance.run_investigation``.
"""

from __future__ import annotations

import dataclasses
import math

import torch
import torch.nn.functional as F

from .batch_invariant_ops import (
    gated_linear_batch_invariant,
    is_batch_invariant_mode_enabled,
    linear_residual_batch_invariant,
)


@dataclasses.dataclass(frozen=True)
class VLAConfig:
    image_size: int = 224
    patch: int = 14
    vis_width: int = 1152
    vis_layers: int = 27
    vis_heads: int = 16
    vis_mlp: int = 4304
    lm_width: int = 2048
    lm_layers: int = 18
    lm_heads: int = 8
    lm_kv_heads: int = 1
    lm_head_dim: int = 256
    lm_mlp: int = 16384
    vocab: int = 257152
    text_tokens: int = 48
    act_width: int = 1024
    act_layers: int = 18
    act_mlp: int = 4096
    chunk: int = 50
    action_dim: int = 32
    flow_steps: int = 10
    dtype: torch.dtype = torch.bfloat16

    @staticmethod
    def full() -> "VLAConfig":
        return VLAConfig()

    @staticmethod
    def tiny() -> "VLAConfig":
        return VLAConfig(image_size=56, patch=14, vis_width=64, vis_layers=2, vis_heads=4,
                         vis_mlp=128, lm_width=128, lm_layers=2, lm_heads=4, lm_kv_heads=1,
                         lm_head_dim=32, lm_mlp=256, vocab=1000, text_tokens=8, act_width=64,
                         act_layers=2, act_mlp=128, chunk=10, action_dim=8, flow_steps=3)


def _w(gen: torch.Generator, *shape: int, device, dtype, scale: float | None = None):
    fan_in = shape[-1] if len(shape) > 1 else shape[0]
    std = scale if scale is not None else 1.0 / math.sqrt(fan_in)
    return (torch.randn(*shape, generator=gen, device=device) * std).to(dtype)


class PiZeroStyleVLA(torch.nn.Module):
    """Inputs: images [B, 3, S, S] in [0, 1], token ids [B, T], noise
    [B, chunk, action_dim].  Output: {"actions": [B, chunk, action_dim],
    "prefix": last prefix hidden state [B, tokens, lm_width]}."""

    def __init__(self, cfg: VLAConfig, device: torch.device | str = "cuda", seed: int = 0):
        super().__init__()
        self.cfg = cfg
        gen = torch.Generator(device=device).manual_seed(seed)
        dt = cfg.dtype
        w = lambda *s, scale=None: torch.nn.Parameter(  # noqa: E731
            _w(gen, *s, device=device, dtype=dt, scale=scale), requires_grad=False
        )
        ones = lambda n: torch.nn.Parameter(  # noqa: E731
            torch.ones(n, device=device, dtype=dt), requires_grad=False
        )
        zeros = lambda n: torch.nn.Parameter(  # noqa: E731
            torch.zeros(n, device=device, dtype=dt), requires_grad=False
        )
        n_patch = (cfg.image_size // cfg.patch) ** 2
        self.patch_w = w(cfg.vis_width, 3, cfg.patch, cfg.patch, scale=0.02)
        self.patch_b = zeros(cfg.vis_width)
        self.vis_pos = w(n_patch, cfg.vis_width, scale=0.02)
        self.vis = torch.nn.ParameterList()
        for _ in range(cfg.vis_layers):
            self.vis.extend([
                ones(cfg.vis_width), zeros(cfg.vis_width),
                w(3 * cfg.vis_width, cfg.vis_width), zeros(3 * cfg.vis_width),
                w(cfg.vis_width, cfg.vis_width), zeros(cfg.vis_width),
                ones(cfg.vis_width), zeros(cfg.vis_width),
                w(cfg.vis_mlp, cfg.vis_width), zeros(cfg.vis_mlp),
                w(cfg.vis_width, cfg.vis_mlp), zeros(cfg.vis_width),
            ])
        self.vis_norm = ones(cfg.vis_width)
        self.vis_norm_b = zeros(cfg.vis_width)
        self.projector = w(cfg.lm_width, cfg.vis_width)
        self.embed = w(cfg.vocab, cfg.lm_width, scale=0.02)
        qkv_lm = (cfg.lm_heads + 2 * cfg.lm_kv_heads) * cfg.lm_head_dim
        self.lm = torch.nn.ParameterList()
        for _ in range(cfg.lm_layers):
            self.lm.extend([
                ones(cfg.lm_width), w(qkv_lm, cfg.lm_width),
                w(cfg.lm_width, cfg.lm_heads * cfg.lm_head_dim),
                ones(cfg.lm_width), w(2 * cfg.lm_mlp, cfg.lm_width), w(cfg.lm_width, cfg.lm_mlp),
            ])
        self.lm_norm = ones(cfg.lm_width)
        # action expert: queries/keys/values in the LM's head layout so that
        # action tokens attend jointly to the prefix keys/values
        self.act_in = w(cfg.act_width, cfg.action_dim + cfg.act_width)
        self.act = torch.nn.ParameterList()
        for _ in range(cfg.act_layers):
            self.act.extend([
                ones(cfg.act_width), w(qkv_lm, cfg.act_width),
                w(cfg.act_width, cfg.lm_heads * cfg.lm_head_dim),
                ones(cfg.act_width), w(2 * cfg.act_mlp, cfg.act_width),
                w(cfg.act_width, cfg.act_mlp),
            ])
        self.act_norm = ones(cfg.act_width)
        self.act_out = w(cfg.action_dim, cfg.act_width)

    # ----------------------------------------------------------------- blocks
    @staticmethod
    def _rms(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        # F.rms_norm: one fused kernel (aten::_fused_rms_norm on CUDA, the
        # library's bio_norm under set_batch_invariant_mode)
        return F.rms_norm(x, (x.shape[-1],), g, 1e-6)

    def _vision(self, images: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        x = F.conv2d(images.to(c.dtype), self.patch_w, self.patch_b, stride=c.patch)
        x = x.flatten(2).transpose(1, 2) + self.vis_pos  # [B, P, W]
        b, n, _ = x.shape
        hd = c.vis_width // c.vis_heads
        p = list(self.vis)
        for i in range(c.vis_layers):
            ln1, ln1b, wqkv, bqkv, wo, bo, ln2, ln2b, w1, b1, w2, b2 = p[12 * i: 12 * i + 12]
            h = F.layer_norm(x, (c.vis_width,), ln1, ln1b)
            q, k, v = F.linear(h, wqkv, bqkv).view(b, n, 3, c.vis_heads, hd).unbind(2)
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                               v.transpose(1, 2))
            x = self._add_linear(x, a.transpose(1, 2).reshape(b, n, c.vis_width), wo, bo)
            h = F.layer_norm(x, (c.vis_width,), ln2, ln2b)
            x = self._add_linear(x, F.gelu(F.linear(h, w1, b1), approximate="tanh"), w2, b2)
        x = F.layer_norm(x, (c.vis_width,), self.vis_norm, self.vis_norm_b)
        return F.linear(x, self.projector)

    def _attn_kv(self, h, wqkv, t):
        c = self.cfg
        b = h.shape[0]
        qkv = F.linear(h, wqkv).view(b, t, c.lm_heads + 2 * c.lm_kv_heads, c.lm_head_dim)
        q = qkv[:, :, : c.lm_heads].transpose(1, 2)
        k = qkv[:, :, c.lm_heads: c.lm_heads + c.lm_kv_heads].transpose(1, 2)
        v = qkv[:, :, c.lm_heads + c.lm_kv_heads:].transpose(1, 2)
        return q, k, v

    @staticmethod
    def _add_linear(r, x, w, b=None):
        """r + F.linear(x, w, b); under the mode one GEMM with the add in its
        epilogue (same rounding steps)."""
        if is_batch_invariant_mode_enabled() and x.is_cuda:
            return linear_residual_batch_invariant(r, x, w, b)
        return r + F.linear(x, w, b)

    def _geglu(self, r, h, w_in, w_out, width):
        """r + down(gelu(gate) * up)."""
        if is_batch_invariant_mode_enabled() and h.is_cuda:
            # the library's fused GeGLU GEMM: same rounding steps as the
            # stock composition below, without the gate/up round trip to HBM
            return self._add_linear(r, gated_linear_batch_invariant(h, w_in, "gelu_tanh"), w_out)
        gate, up = F.linear(h, w_in).split(width, dim=-1)
        return r + F.linear(F.gelu(gate, approximate="tanh") * up, w_out)

    def _prefix(self, image_tokens, ids):
        """Prefix LM.  Returns the final hidden state and, per layer, a joint
        key/value buffer [B, kv_heads, prefix + chunk, head_dim] whose prefix
        part is filled here; the action expert writes its own keys/values
        into the tail at every flow step (no concatenation per step)."""
        c = self.cfg
        x = torch.cat([image_tokens, F.embedding(ids, self.embed)], dim=1)
        x = x * math.sqrt(c.lm_width)
        b, t, _ = x.shape
        p = list(self.lm)
        kv = []
        for i in range(c.lm_layers):
            n1, wqkv, wo, n2, w_in, w_out = p[6 * i: 6 * i + 6]
            q, k, v = self._attn_kv(self._rms(x, n1), wqkv, t)
            kbuf = x.new_empty(b, c.lm_kv_heads, t + c.chunk, c.lm_head_dim)
            vbuf = torch.empty_like(kbuf)
            kbuf[:, :, :t] = k
            vbuf[:, :, :t] = v
            kv.append((kbuf, vbuf))
            a = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
            x = self._add_linear(x, a.transpose(1, 2).reshape(b, t, -1), wo)
            x = self._geglu(x, self._rms(x, n2), w_in, w_out, c.lm_mlp)
        return self._rms(x, self.lm_norm), kv

    def _velocity(self, xt, time, kv):
        c = self.cfg
        b = xt.shape[0]
        half = c.act_width // 2
        freq = torch.exp(-math.log(10000.0) * torch.arange(half, device=xt.device) / half)
        ang = time.float()[:, None] * freq[None]
        temb = torch.cat([ang.sin(), ang.cos()], -1).to(c.dtype)
        h = F.linear(torch.cat([xt, temb[:, None].expand(b, c.chunk, c.act_width)], -1),
                     self.act_in)
        p = list(self.act)
        for i in range(c.act_layers):
            n1, wqkv, wo, n2, w_in, w_out = p[6 * i: 6 * i + 6]
            q, k, v = self._attn_kv(self._rms(h, n1), wqkv, c.chunk)
            kbuf, vbuf = kv[i % len(kv)]
            t_pre = kbuf.shape[2] - c.chunk
            kbuf[:, :, t_pre:] = k
            vbuf[:, :, t_pre:] = v
            a = F.scaled_dot_product_attention(q, kbuf, vbuf, enable_gqa=True)
            h = self._add_linear(h, a.transpose(1, 2).reshape(b, c.chunk, -1), wo)
            h = self._geglu(h, self._rms(h, n2), w_in, w_out, c.act_mlp)
        return F.linear(self._rms(h, self.act_norm), self.act_out)

    def forward(self, images, ids, noise):
        c = self.cfg
        prefix, kv = self._prefix(self._vision(images), ids)
        x = noise.to(c.dtype)
        dt = -1.0 / c.flow_steps
        for s in range(c.flow_steps):
            time = torch.full((x.shape[0],), 1.0 + s * dt, device=x.device)
            x = x + dt * self._velocity(x, time, kv)
        return {"actions": x, "prefix": prefix}


class VLAAdapter:
    """``model_invariance`` adapter: per-sample inputs are seeded synthetic
    (image ~ U[0, 1], ids uniform over the vocabulary, noise ~ N(0, 1))."""

    def __init__(self, cfg: VLAConfig | None = None, device: str = "cuda", seed: int = 0):
        self.cfg = cfg or VLAConfig.tiny()
        self.device = device
        self.seed = seed
        self.name = "pi0-style-vla"

    def load_model(self):
        return PiZeroStyleVLA(self.cfg, self.device, self.seed)

    def load_example_inputs(self, count: int):
        c = self.cfg
        out = []
        for i in range(count):
            g = torch.Generator(device=self.device).manual_seed(1000 + i)
            out.append({
                "images": torch.rand(3, c.image_size, c.image_size, generator=g,
                                     device=self.device),
                "ids": torch.randint(0, c.vocab, (c.text_tokens,), generator=g,
                                     device=self.device),
                "noise": torch.randn(c.chunk, c.action_dim, generator=g, device=self.device),
            })
        return out

    def run_model(self, model, batch):
        return model(batch["images"], batch["ids"], batch["noise"])

    def extract_robot_output(self, output):
        return output
