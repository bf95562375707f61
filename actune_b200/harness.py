"""Benchmark backbones: an OpenVLA-OFT-shaped Llama-2-7B policy with a W4A8 bank.

The reference runs its packed linears inside external OFT / OpenPI models
(actune/models/oft.py, actune/models/pi05.py).  Those are not installable here,
so the benchmark uses a random-init backbone of the same shape:

* Llama-2-7B: 32 decoder layers, hidden 4096, 32 heads x 128, MLP 11008,
  RMSNorm (eps 1e-5), rotary embedding, bf16; fused QKV (4096 -> 12288) and
  fused gate/up (4096 -> 22016) projections, so the four packed linears per
  layer have exactly the Llama-2-7B projection shapes;
* a prefix of 512 vision + 32 prompt tokens followed by 8 x 7 = 56
  parallel-decoded action tokens (600 tokens per call), whose final states go
  through a small bf16 action head to an [8, 7] action chunk.

Every projection is a bank target, installed with ``install_bank`` (so it runs
the packed-integer path) under a W4A8-average ``SharedBank`` with two binary
switchable matrices.  Attention uses torch SDPA; norms, rotary embedding and
the gated activation use the glue kernels of include/actune_b200_harness.h.
"""
from __future__ import annotations

import ctypes

import numpy as np

import torch
import torch.nn.functional as F

from . import _lib
from .kernels.grouped import share_quantized, shared_activation_active
from .layers import expected_version_bytes, install_bank
from .precision import CONFIGURATIONS, SharedBank

_H = None


def _hlib():
    global _H
    if _H is None:
        L = _lib.lib()
        p, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.actune_harness_rmsnorm.argtypes = [p, p, p, p, p, i64, i64, ctypes.c_float, i32, p]
        L.actune_harness_rmsnorm.restype = i32
        L.actune_harness_rope.argtypes = [p, p, p, i64, i32, i32, i32, p]
        L.actune_harness_rope.restype = i32
        L.actune_harness_gated_act.argtypes = [p, p, i64, i64, i32, p]
        L.actune_harness_gated_act.restype = i32
        L.actune_harness_rmsnorm_q.argtypes = [p, p, p, p, p, i64, i64, ctypes.c_float, i32, i32, i32, p, p, p]
        L.actune_harness_rmsnorm_q.restype = i32
        L.actune_harness_gated_act_q.argtypes = [p, p, i64, i64, i32, i32, i32, p, p, p]
        L.actune_harness_gated_act_q.restype = i32
        L.actune_harness_rope_cache.argtypes = [p, p, p, i64, i32, i32, p, i64, i64, i64, p]
        L.actune_harness_rope_cache.restype = i32
        _H = L
    return _H


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _s(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def rmsnorm(x, weight, eps, residual=None, gemma=False, quant_bits=None, codes8=False):
    """(normed, new_residual): fused residual add + RMSNorm over the last dim.

    With ``quant_bits`` the kernel also writes the group-64 activations of the
    normed output (packed, or one int8 code each with ``codes8``) and offers them
    to the active shared activation scope, so the next projection does not launch
    its own quantizer."""
    x = x.contiguous()
    out = torch.empty_like(x)
    res_out = torch.empty_like(x) if residual is not None else None
    T, D = x.numel() // x.shape[-1], x.shape[-1]
    if quant_bits and D % 256 == 0 and D <= 8192:
        width = 8 if codes8 else quant_bits
        packed = torch.empty((T, D * width // 8), device=x.device, dtype=torch.uint8)
        scales = torch.empty((T, D // 64), device=x.device, dtype=torch.float32)
        _lib.check(_hlib().actune_harness_rmsnorm_q(_p(x), _p(residual), _p(weight), _p(out), _p(res_out), T, D,
                                                     float(eps), 1 if gemma else 0, int(quant_bits),
                                                     1 if codes8 else 0, _p(packed),
                                                     _p(scales), _s(x)), "rmsnorm")
        share_quantized(out.view(T, D), quant_bits, packed, scales, codes8)
    else:
        _lib.check(_hlib().actune_harness_rmsnorm(_p(x), _p(residual), _p(weight), _p(out), _p(res_out), T, D,
                                                   float(eps), 1 if gemma else 0, _s(x)), "rmsnorm")
    return out, (res_out if residual is not None else x)


def rope_(qkv, cos, sin, hq, hkv, dh):
    T = qkv.numel() // qkv.shape[-1]
    _lib.check(_hlib().actune_harness_rope(_p(qkv), _p(cos), _p(sin), T, hq, hkv, dh, _s(qkv)), "rope")
    return qkv


def rope_cache_(qkv, cos, sin, hq, dh, cache, seq, offset):
    """rope_ for one key/value head that also writes each token's rotated key and
    its value into ``cache`` [B, Tc, 2, dh] at positions offset .. offset + seq - 1."""
    T = qkv.numel() // qkv.shape[-1]
    _lib.check(_hlib().actune_harness_rope_cache(_p(qkv), _p(cos), _p(sin), T, hq, dh, _p(cache), seq,
                                                 _cache_pitch(cache, dh), offset, _s(qkv)), "rope_cache")
    return qkv


def _cache_pitch(cache, dh):
    """Positions between consecutive sequences of a [B, T, 2, dh] cache view whose
    rows are contiguous (a slice of a longer buffer keeps the buffer's pitch)."""
    if cache.dim() != 4 or cache.shape[2:] != (2, dh) or cache.stride()[1:] != (2 * dh, dh, 1) or \
            cache.stride(0) % (2 * dh):
        raise ValueError("the cache must be [B, T, 2, head_dim] with contiguous rows")
    return cache.stride(0) // (2 * dh) if cache.shape[0] > 1 else cache.shape[1]


def gated_act(gu, gelu=False, quant_bits=None, codes8=False):
    """act(gate) * up for gu = [gate | up]; with ``quant_bits`` also the group-64
    activations of the result (packed, or int8 codes with ``codes8``), offered to
    the shared activation scope."""
    I = gu.shape[-1] // 2
    T = gu.numel() // gu.shape[-1]
    gu = gu.contiguous()
    out = torch.empty(*gu.shape[:-1], I, device=gu.device, dtype=gu.dtype)
    if quant_bits and I % 64 == 0:
        width = 8 if codes8 else quant_bits
        packed = torch.empty((T, I * width // 8), device=gu.device, dtype=torch.uint8)
        scales = torch.empty((T, I // 64), device=gu.device, dtype=torch.float32)
        _lib.check(_hlib().actune_harness_gated_act_q(_p(gu), _p(out), T, I, 1 if gelu else 0, int(quant_bits),
                                                       1 if codes8 else 0, _p(packed), _p(scales), _s(gu)),
                   "gated_act")
        share_quantized(out.view(T, I), quant_bits, packed, scales, codes8)
    else:
        _lib.check(_hlib().actune_harness_gated_act(_p(gu), _p(out), T, I, 1 if gelu else 0, _s(gu)), "gated_act")
    return out


def input_format(module, rows):
    """{"quant_bits": A, "codes8": bool}: how `module` quantizes an input of `rows`
    token rows, when the input reaches its quantizer unchanged (a grouped bank
    module without K padding or a runtime channel scale, inside an active shared
    activation scope); else {} (the glue then writes no activations)."""
    if not shared_activation_active() or not hasattr(module, "active_backend"):
        return {}
    if getattr(module, "padding", 0) or getattr(module, "input_scale", None) is not None:
        return {}
    bits, codes8 = module.active_backend().activation_format(rows)
    return {"quant_bits": bits, "codes8": codes8}


def rope_tables(T, dh, theta, device):
    inv = 1.0 / (theta ** (torch.arange(0, dh, 2, device=device, dtype=torch.float32) / dh))
    ang = torch.arange(T, device=device, dtype=torch.float32)[:, None] * inv[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()


class DecoderLayer(torch.nn.Module):
    """Pre-norm decoder layer with fused QKV and gate/up projections (Llama or Gemma flavour)."""

    def __init__(self, hidden, heads, kv_heads, head_dim, mlp, eps, gemma, device, dtype):
        super().__init__()
        self.hidden, self.heads, self.kv_heads, self.head_dim, self.mlp = hidden, heads, kv_heads, head_dim, mlp
        self.eps, self.gemma = eps, gemma
        kw = dict(device=device, dtype=dtype)
        self.input_norm = torch.nn.Parameter(torch.ones(hidden, **kw) if not gemma else torch.zeros(hidden, **kw))
        self.post_norm = torch.nn.Parameter(torch.ones(hidden, **kw) if not gemma else torch.zeros(hidden, **kw))
        self.qkv_proj = torch.nn.Linear(hidden, (heads + 2 * kv_heads) * head_dim, bias=False, **kw)
        self.o_proj = torch.nn.Linear(heads * head_dim, hidden, bias=False, **kw)
        self.gate_up_proj = torch.nn.Linear(hidden, 2 * mlp, bias=False, **kw)
        self.down_proj = torch.nn.Linear(mlp, hidden, bias=False, **kw)

    def forward(self, x, residual, cos, sin, causal=True, batch=1, cache=None, offset=0):
        """(x, residual) -> (mlp output, new residual stream), pre-norm.

        x holds `batch` independent sequences of T tokens as [batch * T, hidden]
        rows (the projections see all rows at once; attention stays within each
        sequence); cos / sin hold the rotary table of every row; `causal`: causal
        attention within the call (bidirectional otherwise).

        `cache`: a key/value buffer [batch, T_cache, 2, head_dim] (one KV head) for
        this layer.  The call's rotated keys and values are written at positions
        [offset, offset + T) with one copy, and attention runs over positions
        [0, offset + T) -- the prefix cached by earlier calls plus this call."""
        rows = x.shape[0]
        B, T = batch, rows // batch
        h, residual = rmsnorm(x, self.input_norm, self.eps, residual, self.gemma,
                              **input_format(self.qkv_proj, rows))
        qkv = self.qkv_proj(h)
        qd, kvd = self.heads * self.head_dim, self.kv_heads * self.head_dim
        if cache is None:
            rope_(qkv, cos, sin, self.heads, self.kv_heads, self.head_dim)
            k = qkv[:, qd:qd + kvd].view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
            v = qkv[:, qd + kvd:].view(B, T, self.kv_heads, self.head_dim).transpose(1, 2)
        else:
            if self.kv_heads != 1:
                raise ValueError("the key/value cache holds one KV head")
            # One launch rotates and writes the call's keys and values into the cache.
            rope_cache_(qkv, cos, sin, self.heads, self.head_dim, cache, T, offset)
            k = cache[:, :offset + T, 0].unsqueeze(1)
            v = cache[:, :offset + T, 1].unsqueeze(1)
        q = qkv[:, :qd].view(B, T, self.heads, self.head_dim).transpose(1, 2)
        attn = F.scaled_dot_product_attention(q, k, v, is_causal=causal and offset == 0,
                                              enable_gqa=self.kv_heads != self.heads)
        attn = attn.transpose(1, 2).reshape(rows, self.heads * self.head_dim)
        x = self.o_proj(attn)
        h, residual = rmsnorm(x, self.post_norm, self.eps, residual, self.gemma,
                              **input_format(self.gate_up_proj, rows))
        x = self.down_proj(gated_act(self.gate_up_proj(h), gelu=self.gemma, **input_format(self.down_proj, rows)))
        return x, residual


class OFTBackbone(torch.nn.Module):
    """OpenVLA-OFT-shaped Llama-2-7B backbone + L1-regression-style action head."""

    def __init__(self, layers=32, hidden=4096, heads=32, mlp=11008, tokens=600, action_tokens=56,
                 chunk=(8, 7), device="cuda", dtype=torch.bfloat16, seed=0):
        super().__init__()
        g = torch.Generator(device=device).manual_seed(seed)
        self.tokens, self.action_tokens, self.chunk = tokens, action_tokens, chunk
        self.layers = torch.nn.ModuleList(
            [DecoderLayer(hidden, heads, heads, hidden // heads, mlp, 1e-5, False, device, dtype) for _ in range(layers)])
        with torch.no_grad():
            for layer in self.layers:
                for lin in (layer.qkv_proj, layer.o_proj, layer.gate_up_proj, layer.down_proj):
                    lin.weight.normal_(0.0, 0.02, generator=g)
        self.final_norm = torch.nn.Parameter(torch.ones(hidden, device=device, dtype=dtype))
        self.head1 = torch.nn.Linear(hidden, hidden, device=device, dtype=dtype)
        self.head2 = torch.nn.Linear(hidden, 1, device=device, dtype=dtype)
        with torch.no_grad():
            for lin in (self.head1, self.head2):
                lin.weight.normal_(0.0, 0.02, generator=g)
                lin.bias.zero_()
        cos, sin = rope_tables(tokens, hidden // heads, 10000.0, device)
        self.register_buffer("rope_cos", cos)
        self.register_buffer("rope_sin", sin)

    def forward(self, embeds):
        """embeds [tokens, hidden] bf16 -> actions [chunk] fp32."""
        x, residual = embeds, None
        for layer in self.layers:
            x, residual = layer(x, residual, self.rope_cos, self.rope_sin)
        h, _ = rmsnorm(x, self.final_norm, 1e-5, residual)
        a = h[-self.action_tokens:]
        a = self.head2(F.gelu(self.head1(a)))
        return a.float().reshape(self.chunk)


def projection_names(model, stacks=("layers",)):
    names = []
    for stack in stacks:
        for i in range(len(getattr(model, stack))):
            for proj in ("qkv_proj", "o_proj", "gate_up_proj", "down_proj"):
                names.append(f"{stack}.{i}.{proj}")
    return names


def build_bank(model, tokens, base, alternate, switchable, stacks=("layers",)):
    """Synthetic SharedBank: every projection in mode `base`, two binary switchable
    matrices that take mode `alternate` in the configurations that select them
    (q11: neither, q10: the second, q01: the first, q00: both).  `tokens` maps a
    stack name to the token rows one request feeds its projections."""
    names = projection_names(model, stacks)
    shapes = {n: [model.get_submodule(n).out_features, model.get_submodule(n).in_features] for n in names}
    counts = {n: tokens[n.split(".")[0]] * shapes[n][1] for n in names}
    base_cfg = {n: base for n in names}
    a, b = switchable
    configurations = {
        "q11": dict(base_cfg),
        "q10": {**base_cfg, b: alternate},
        "q01": {**base_cfg, a: alternate},
        "q00": {**base_cfg, a: alternate, b: alternate},
    }
    version_bytes = {n: {m: expected_version_bytes(shapes[n][0], shapes[n][1], int(m[1]), int(m[3]))
                         for m in {c[n] for c in configurations.values()}} for n in names}
    groups = {}
    for n in names:
        groups.setdefault(n.split(".")[0] + "." + n.split(".")[-1], []).append(n)
    resident = sum(version_bytes[n][m] for n in names for m in version_bytes[n])
    bank = SharedBank(configurations=configurations, shapes=shapes, activation_elements=counts,
                      shape_groups=list(groups.values()), version_bytes=version_bytes, budget=base,
                      storage_limit=resident + 1024)
    clips = {n: {m: None for m in version_bytes[n]} for n in names}
    return bank.validate(), clips


def build_w4a8_bank(model, tokens, switchable=("layers.0.down_proj", "layers.1.down_proj")):
    """W4A8-average bank of the OFT backbone: every projection W4A8, two binary
    switchable matrices (W4A8 / W2A8), four distinct configurations."""
    return build_bank(model, {"layers": tokens}, "w4a8", "w2a8", switchable)


def make_oft_policy(layers=32, tokens=600, device="cuda", seed=0, decoded=True):
    """Build the backbone, install the packed bank (frees the bf16 weights) and
    return (model, runtime).  ``decoded``: also keep int8 weight codes for the tile
    GEMM (``BankRuntime.decode_weights``; bit-identical outputs)."""
    model = OFTBackbone(layers=layers, tokens=tokens, device=device, seed=seed)
    bank, clips = build_w4a8_bank(model, tokens)
    runtime = install_bank(model, bank, clips)
    runtime.decoded_bytes = runtime.decode_weights() if decoded else 0
    torch.cuda.synchronize()
    return model, runtime


def config_cycle():
    """Per-call precision order used by the benchmark: q00 -> q01 -> q11 -> q10."""
    return ("q00", "q01", "q11", "q10")


assert set(config_cycle()) == set(CONFIGURATIONS)


# ---------------------------------------------------------------------------- pi0.5-shaped policy
class Pi05Backbone(torch.nn.Module):
    """pi0.5-shaped VLA policy: a Gemma-2B-like VLM over the prefix and a
    Gemma-300M-like action expert run through ten flow-matching Euler steps.

    * VLM: 18 layers, hidden 2048, 8 query heads / 1 KV head of 256, MLP 16384,
      RMSNorm (1 + w), tanh-GELU gated MLP; the 256 image + 48 text prefix tokens
      attend to one another bidirectionally, and every layer's rotated keys and
      values are kept in a prefix cache.
    * Action expert: 18 layers, width 1024, the same head layout (queries 8 x 256,
      one KV head), MLP 4096.  Each layer of a denoise step attends to its VLM
      layer's prefix cache plus the 50 action tokens' own keys and values.
    * A denoise step embeds the noisy [50, 32] action chunk and the flow time,
      runs the expert and projects back to a velocity; the sampler follows the
      reference's frozen ten-step loop (actune/models/pi05.py:28-37): the time
      tensor starts at float32(1) and adds float32(-1/10) in place after every
      step, x_t = x_t + dt * v_t.

    The image tokens are random bf16 embeddings of the stated count (no vision
    encoder is specified); every projection of both stacks is a bank target."""

    def __init__(self, vlm_layers=18, vlm_hidden=2048, vlm_mlp=16384, expert_layers=18, expert_hidden=1024,
                 expert_mlp=4096, heads=8, kv_heads=1, head_dim=256, prefix_tokens=304, horizon=50, action_dim=32,
                 steps=10, max_batch=1, state_dim=0, device="cuda", dtype=torch.bfloat16, seed=0):
        super().__init__()
        if vlm_layers != expert_layers:
            raise ValueError("the action expert attends to the VLM layer of the same depth")
        g = torch.Generator(device=device).manual_seed(seed)
        kw = dict(device=device, dtype=dtype)
        self.prefix_tokens, self.horizon, self.action_dim, self.steps = prefix_tokens, horizon, action_dim, steps
        self.max_batch, self.state_dim = max_batch, state_dim
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.vlm = torch.nn.ModuleList([DecoderLayer(vlm_hidden, heads, kv_heads, head_dim, vlm_mlp, 1e-6, True,
                                                     device, dtype) for _ in range(vlm_layers)])
        self.expert = torch.nn.ModuleList([DecoderLayer(expert_hidden, heads, kv_heads, head_dim, expert_mlp, 1e-6,
                                                        True, device, dtype) for _ in range(expert_layers)])
        self.action_in = torch.nn.Linear(action_dim, expert_hidden, **kw)
        self.time_in = torch.nn.Linear(expert_hidden, expert_hidden, **kw)
        self.time_out = torch.nn.Linear(expert_hidden, expert_hidden, **kw)
        self.action_out = torch.nn.Linear(expert_hidden, action_dim, **kw)
        self.final_norm = torch.nn.Parameter(torch.zeros(expert_hidden, **kw))
        # Proprioceptive state, when the policy is given one: projected and added to
        # every action token of its environment.
        self.state_in = torch.nn.Linear(state_dim, expert_hidden, **kw) if state_dim else None
        with torch.no_grad():
            for layer in list(self.vlm) + list(self.expert):
                for lin in (layer.qkv_proj, layer.o_proj, layer.gate_up_proj, layer.down_proj):
                    lin.weight.normal_(0.0, 0.02, generator=g)
            for lin in (self.action_in, self.time_in, self.time_out, self.action_out, self.state_in):
                if lin is not None:
                    lin.weight.normal_(0.0, 0.02, generator=g)
                    lin.bias.zero_()
        cos, sin = rope_tables(prefix_tokens + horizon, head_dim, 10000.0, device)
        self.register_buffer("rope_cos", cos)
        self.register_buffer("rope_sin", sin)
        half = expert_hidden // 2
        freqs = torch.exp(-torch.arange(half, device=device, dtype=torch.float32) * (torch.log(torch.tensor(
            10000.0, device=device)) / half))
        self.register_buffer("time_freqs", freqs)
        if kv_heads != 1:
            raise ValueError("the pi0.5 layout has one KV head")
        # Per VLM layer: keys and values of the prefix, then room for the action
        # tokens of a denoise step (written by the expert layer of the same depth).
        cache = torch.zeros(vlm_layers, max_batch, prefix_tokens + horizon, 2, head_dim, **kw)
        self.register_buffer("prefix_cache", cache)
        self._rope_rows = {}

    def _rope(self, b, start, count):
        """Rotary tables for b sequences of `count` positions from `start`, one row per token."""
        key = (b, start, count)
        if key not in self._rope_rows:
            self._rope_rows[key] = (self.rope_cos[start:start + count].repeat(b, 1).contiguous(),
                                    self.rope_sin[start:start + count].repeat(b, 1).contiguous())
        return self._rope_rows[key]

    def prefix(self, embeds):
        """VLM pass over the prefix tokens ([304, 2048], or [b, 304, 2048] for b
        environments): fills the first b entries of the prefix cache."""
        b = 1 if embeds.dim() == 2 else embeds.shape[0]
        if b > self.max_batch:
            raise ValueError("batch larger than the prefix cache")
        T = self.prefix_tokens
        x, residual = embeds.reshape(b * T, -1), None
        cos, sin = self._rope(b, 0, T)
        for i, layer in enumerate(self.vlm):
            x, residual = layer(x, residual, cos, sin, causal=False, batch=b, cache=self.prefix_cache[i, :b, :T],
                                offset=0)
        return self.prefix_cache

    def velocity(self, x_t, time, state=None):
        """v_t for the noisy chunk x_t ([50, 32], or [b, 50, 32]; fp32) at flow time
        `time` (0-dim fp32), attending to the first b prefix caches."""
        b = 1 if x_t.dim() == 2 else x_t.shape[0]
        T0, T = self.prefix_tokens, self.horizon
        dtype = self.action_in.weight.dtype
        ang = time * self.time_freqs
        temb = torch.cat([ang.sin(), ang.cos()]).to(dtype)
        tvec = self.time_out(F.silu(self.time_in(temb)))
        x = self.action_in(x_t.reshape(b * T, -1).to(dtype)) + tvec
        if state is not None and self.state_in is not None:
            x = (x.view(b, T, -1) + self.state_in(state.to(dtype))[:, None, :]).reshape(b * T, -1)
        residual = None
        cos, sin = self._rope(b, T0, T)
        for i, layer in enumerate(self.expert):
            x, residual = layer(x, residual, cos, sin, causal=False, batch=b, cache=self.prefix_cache[i, :b],
                                offset=T0)
        h, _ = rmsnorm(x, self.final_norm, 1e-6, residual, gemma=True)
        return self.action_out(h).float().view(x_t.shape)

    def denoise_step(self, x_t, time, dt, state=None):
        """One Euler step of the frozen sampler: (x_t + dt * v_t, time + dt)."""
        v_t = self.velocity(x_t, time, state)
        return x_t + dt * v_t, time + dt


def make_pi05_policy(device="cuda", seed=0, decoded=True, **shape):
    """Build the pi0.5-shaped backbone and install its W4A4-average bank (every
    projection of both stacks W4A4, two binary switchable matrices W4A4 / W2A4).
    ``decoded`` as for ``make_oft_policy``."""
    model = Pi05Backbone(device=device, seed=seed, **shape)
    tokens = {"vlm": model.prefix_tokens, "expert": model.horizon * model.steps}
    bank, clips = build_bank(model, tokens, "w4a4", "w2a4", ("vlm.0.down_proj", "expert.0.down_proj"),
                             stacks=("vlm", "expert"))
    runtime = install_bank(model, bank, clips)
    runtime.decoded_bytes = runtime.decode_weights() if decoded else 0
    torch.cuda.synchronize()
    return model, runtime


def sample_pi05(model, prefix_call, step_call, embeds, noise, state=None):
    """One action chunk: the prefix pass, then the frozen ten-step Euler loop with a
    float32 time tensor that starts at 1 and adds float32(-1/steps) per step.
    `prefix_call` / `step_call` are the model's prefix / denoise_step, or their
    graph-replayed wrappers (one CUDA graph per step shape)."""
    prefix_call(embeds)
    # The same float32 values as torch.tensor(-1 / steps) and torch.tensor(1.0), made
    # by fill kernels: a tensor built from a host scalar is a blocking host-to-device
    # copy, which would stall the host here until the prefix has run.
    dt = torch.full((), -1.0 / model.steps, dtype=torch.float32, device=noise.device)
    time = torch.full((), 1.0, dtype=torch.float32, device=noise.device)
    x_t = noise
    for _ in range(model.steps):
        x_t, time = step_call(x_t, time, dt) if state is None else step_call(x_t, time, dt, state)
    return x_t


# ---------------------------------------------------------------------------- pi0.5 serving replica
class Pi05Serving:
    """One serving replica of the pi0.5-shaped policy: `envs` environments, each
    request a 224 x 224 x 3 uint8 image and a 14-dim proprioceptive state.

    The image goes through a patch stem (14 x 14 patches -> 256 tokens, one bf16
    linear 588 -> 2048; no vision encoder is specified) and is followed by 48
    prompt-token embeddings; the state is projected onto the action tokens.  A
    group of environments sharing a configuration is padded to a batch bucket and
    runs one prefix graph and ten denoise-step graphs (one CUDA graph per bucket,
    step shape and configuration)."""

    PATCH, IMAGE, TEXT = 14, 224, 48

    def __init__(self, envs=16, buckets=(4, 8, 16), seed=0, device="cuda", **shape):
        from .graph import GraphReplay
        self.envs, self.buckets, self.device = envs, tuple(buckets), device
        self.model, self.runtime = make_pi05_policy(device=device, seed=seed, max_batch=max(buckets), state_dim=14,
                                                    **shape)
        m = self.model
        hidden = m.vlm[0].hidden
        g = torch.Generator(device=device).manual_seed(seed + 1)
        self.stem = torch.nn.Linear(self.PATCH * self.PATCH * 3, hidden, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            self.stem.weight.normal_(0.0, 0.02, generator=g)
            self.stem.bias.zero_()
        self.text = (torch.randn(self.TEXT, hidden, device=device, generator=g) * 0.5).bfloat16()
        self.patches = (self.IMAGE // self.PATCH) ** 2
        if self.patches + self.TEXT != m.prefix_tokens:
            raise ValueError("prefix tokens must be 256 image patches + 48 prompt tokens")
        self.prefix = GraphReplay(self._prefix, self.runtime.modules, shared_a8=True, max_graphs=4 * len(buckets))
        self.step = GraphReplay(m.denoise_step, self.runtime.modules, shared_a8=True, max_graphs=4 * len(buckets))
        self.prefix.enabled = self.step.enabled = True
        gn = torch.Generator(device=device).manual_seed(seed + 2)
        self.noise = torch.randn(max(buckets), m.horizon, m.action_dim, device=device, generator=gn)

    def _prefix(self, images):
        """uint8 images [b, 224, 224, 3] -> the VLM prefix pass over [b, 304, hidden]."""
        b, P = images.shape[0], self.PATCH
        x = images.view(b, self.IMAGE // P, P, self.IMAGE // P, P, 3).permute(0, 1, 3, 2, 4, 5)
        x = x.reshape(b, self.patches, P * P * 3).to(torch.bfloat16) * (2.0 / 255.0) - 1.0
        tokens = torch.cat([self.stem(x), self.text.expand(b, -1, -1)], dim=1)
        return self.model.prefix(tokens)

    def chunk(self, config, images, states, rows, size):
        """Actions [len(rows), 50, 32] (device) for the environments `rows` of the
        device batches images [envs, ...] / states [envs, 14], padded to `size`."""
        from .precision import precision_profile
        idx = torch.as_tensor(np.pad(rows, (0, size - len(rows)), mode="edge"), device=self.device)
        with precision_profile(config), torch.inference_mode():
            out = sample_pi05(self.model, self.prefix, self.step, images.index_select(0, idx),
                              self.noise[:size], states.index_select(0, idx))
        return out[: len(rows)]

    def release(self):
        self.prefix.release()
        self.step.release()
