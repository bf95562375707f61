"""GPU tests of the reference-facing API on top of the sm_100a kernels.

Mirrors the reference's kernel test (tests/test_kernels.py:30-49: all nine
pairs through GroupedLinear at (1,64,32) and (17,128,96) against the float
dequantized formula, rtol = atol = 0.02) and adds bit-exact checks against the
oracle, K padding, precision switching, install_bank's storage audit,
GraphReplay, the tuner, the one-call workspace entry point and the shared
quantization scope."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O

pytestmark = pytest.mark.gpu
PAIRS = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module", autouse=True)
def device_error_word_clean():
    from actune_b200 import _lib
    _lib.device_error(reset=True)
    yield
    assert _lib.device_error()[0] == 0


def test_all_nine_pairs_against_the_reference_formula():
    """The reference's kernel test, formula evaluated on the CPU: torch's CUDA
    division by a Python scalar multiplies by the reciprocal, so evaluating
    activation_reference on CUDA can put an A4 scale 1 ulp away from the IEEE
    quotient the reference defines (its CPU semantics, pinned by the goldens)."""
    from actune_b200.kernels.grouped import GroupedLinear
    from actune_b200.kernels.quantizers import weight_codes
    torch.manual_seed(7)
    for m, k, n in [(1, 64, 32), (17, 128, 96)]:
        linear = torch.nn.Linear(k, n, bias=True, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        for w, a in PAIRS:
            with torch.inference_mode():
                backend = GroupedLinear(linear, w, a, None)
                actual = backend(x).cpu()
                q, scale = weight_codes(linear.weight, w, a)
                expected = F.linear(O.activation_reference(x.cpu(), a), q.cpu().float() * scale.cpu()[:, None],
                                    linear.bias.detach().cpu().float()).to(x.dtype)
            torch.testing.assert_close(actual, expected, rtol=0.02, atol=0.02)
            assert actual.shape == (m, n)


@pytest.mark.parametrize("w,a", [(4, 8), (2, 4), (8, 4), (4, 4)])
def test_grouped_linear_bit_exact_against_oracle(w, a):
    from actune_b200.kernels.grouped import GroupedLinear
    torch.manual_seed(11)
    linear = torch.nn.Linear(512, 200, bias=True, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(3, 45, 512, device="cuda", dtype=torch.bfloat16)
    layer = GroupedLinear(linear, w, a, None)
    y = layer(x)
    assert y.shape == (3, 45, 200) and y.dtype == torch.bfloat16
    pa, as_ = O.quantize_group64(bits(x.reshape(-1, 512)), a)
    bias = layer.bias.float().cpu().numpy()
    ref = O.packed_linear(pa, as_, layer.packed_weight.cpu().numpy(), layer.weight_scale.cpu().numpy(), bias,
                          512, w, a, fma=True)
    assert np.array_equal(bits(y.reshape(-1, 200)), O.to_bf16_bits(ref))
    # buffers: reference names, shapes and dtypes
    assert layer.packed_weight.shape == (200, 512 * w // 8) and layer.packed_weight.dtype == torch.uint8
    assert layer.weight_scale.shape == (200,) and layer.weight_scale.dtype == torch.float32
    assert layer.bias.dtype == (torch.float32 if a == 4 else torch.bfloat16)


def test_padded_linear_switches_precision_and_counts():
    from actune_b200.kernels.grouped import GroupedPaddedLinear
    from actune_b200.precision import precision_profile
    torch.manual_seed(3)
    linear = torch.nn.Linear(192, 64, bias=False, device="cuda", dtype=torch.bfloat16)  # K padded to 256
    assignments = {"q00": "w2a8", "q01": "w2a8", "q10": "w4a8", "q11": "w4a8"}
    layer = GroupedPaddedLinear(linear, assignments, "q11", {"w2a8": None, "w4a8": None})
    assert layer.padding == 64 and set(layer.backends) == {"w2a8", "w4a8"}
    x = torch.randn(5, 192, device="cuda", dtype=torch.bfloat16)
    y_default = layer(x)
    with precision_profile("q00"):
        y00 = layer(x)
    with precision_profile("q11"):
        y11 = layer(x)
    assert torch.equal(y_default, y11) and not torch.equal(y00, y11)
    xp = F.pad(x, (0, 64))
    assert torch.equal(y00, layer.backends["w2a8"](xp))
    assert layer.calls == 3 and layer.input_elements == 3 * x.numel()
    assert layer.weight.dtype == torch.bfloat16


def tiny_model(seed=0):
    torch.manual_seed(seed)
    m = torch.nn.Sequential(torch.nn.Linear(128, 256, bias=True), torch.nn.GELU(),
                            torch.nn.Linear(256, 128, bias=False)).cuda().to(torch.bfloat16)
    return m


def tiny_bank(model):
    from actune_b200.layers import expected_version_bytes
    from actune_b200.precision import SharedBank
    shapes = {"0": [256, 128], "2": [128, 256]}
    counts = {"0": 4 * 128, "2": 4 * 256}
    cfg = {"q11": {"0": "w4a8", "2": "w4a8"}, "q10": {"0": "w4a8", "2": "w2a8"},
           "q01": {"0": "w2a8", "2": "w4a8"}, "q00": {"0": "w2a8", "2": "w2a8"}}
    vb = {"0": {m: expected_version_bytes(256, 128, int(m[1]), int(m[3]), torch.bfloat16) for m in ("w4a8", "w2a8")},
          "2": {m: expected_version_bytes(128, 256, int(m[1]), int(m[3])) for m in ("w4a8", "w2a8")}}
    return SharedBank(cfg, shapes, counts, [["0"], ["2"]], vb, "w4a8", 10 ** 7)


def test_install_bank_audits_storage_and_runs():
    from actune_b200.layers import ResidentLinear, install_bank
    from actune_b200.precision import precision_profile
    model = tiny_model()
    x = torch.randn(4, 128, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        ref = model(x)
    bank = tiny_bank(model)
    clips = {"0": {"w4a8": None, "w2a8": 0.9}, "2": {"w4a8": None, "w2a8": None}}
    runtime = install_bank(model, bank, clips)
    assert isinstance(model[0], ResidentLinear) and isinstance(model[2], ResidentLinear)
    runtime.before()
    with precision_profile("q11"):
        y = model(x)
    rel = float((y.float() - ref.float()).norm() / ref.float().norm().detach())
    assert rel < 0.15, rel  # 4-bit weights (and 2-bit where the bank says so): close to the bf16 model
    metrics = runtime.audit("q11")
    assert metrics["activation_bits"] == 8 and metrics["weight_bits"] <= 4
    bad = tiny_bank(model)
    bad.version_bytes["0"]["w4a8"] += 1
    with pytest.raises(ValueError, match="storage differs"):
        install_bank(tiny_model(), bad, clips)


def test_resident_linear_channel_scale():
    from actune_b200.layers import ResidentLinear
    torch.manual_seed(5)
    linear = torch.nn.Linear(128, 64, bias=False, device="cuda", dtype=torch.bfloat16)
    scale = torch.rand(128, device="cuda") + 0.5
    layer = ResidentLinear(linear, {q: "w8a8" for q in ("q00", "q01", "q10", "q11")}, {"w8a8": None}, scale)
    x = torch.randn(8, 128, device="cuda", dtype=torch.bfloat16)
    y = layer(x)
    ref = linear(x)
    assert float((y.float() - ref.float()).norm() / ref.float().norm()) < 0.05
    with pytest.raises(ValueError, match="channel scale"):
        ResidentLinear(linear, {"q11": "w8a8"}, {"w8a8": None}, -scale)


def test_graph_replay_matches_eager_per_precision():
    from actune_b200.graph import GraphReplay
    from actune_b200.layers import install_bank
    from actune_b200.precision import precision_profile
    model = tiny_model(1)
    runtime = install_bank(model, tiny_bank(model), {"0": {"w4a8": None, "w2a8": None},
                                                     "2": {"w4a8": None, "w2a8": None}})
    x = torch.randn(4, 128, device="cuda", dtype=torch.bfloat16)
    eager = {}
    with torch.inference_mode():
        for q in ("q00", "q01", "q10", "q11"):
            with precision_profile(q):
                eager[q] = model(x).clone()
    replay = GraphReplay(model, runtime.modules, max_graphs=3)
    replay.enabled = True
    runtime.before()
    for q in ("q00", "q01", "q10", "q11", "q00"):
        with precision_profile(q), torch.inference_mode():
            out = replay(x).clone()
        assert torch.equal(out, eager[q]), q
    assert len(replay.graphs) == 3 and replay.fallbacks == 1 and replay.replays == 4
    # counters: 5 calls recorded on every layer (replays add the captured counts)
    assert all(m.calls == 5 for m in runtime.modules.values())
    replay.release()


def test_extension_linear_signature():
    from actune_b200 import ops
    from actune_b200.kernels.grouped import extension
    torch.manual_seed(2)
    a_src = torch.randn(9, 256, device="cuda", dtype=torch.bfloat16)
    codes, ws = ops.weight_codes((torch.randn(64, 256, device="cuda") * 0.02).bfloat16(), 4, 4)
    pw = ops.pack_rows(codes, 4)
    pa, as_ = ops.quantize_group64(a_src, 4)
    empty = torch.empty(0, device="cuda", dtype=torch.float32)
    y = extension().linear(pa, as_, pw, ws, empty, a_src, 4, 4)
    y1 = extension().linear(pa, as_, pw, ws, empty, a_src, 4, 4, 1)
    assert y.shape == (9, 64) and y.dtype == torch.bfloat16 and torch.equal(y, y1)
    with pytest.raises(RuntimeError):
        extension().linear(pa.cpu(), as_, pw, ws, empty, a_src, 4, 4)


def test_tuned_forward_is_bit_identical():
    from actune_b200.kernels import tuning
    from actune_b200.kernels.grouped import GroupedLinear
    from types import MethodType
    torch.manual_seed(9)
    linear = torch.nn.Linear(1024, 512, bias=True, device="cuda", dtype=torch.bfloat16)
    layer = GroupedLinear(linear, 4, 8, None)
    x = torch.randn(70, 1024, device="cuda", dtype=torch.bfloat16)
    y0 = layer(x)
    layer.forward = MethodType(tuning.grouped_forward, layer)
    y1 = layer(x)
    assert torch.equal(y0, y1)
    key = ("grouped", 4, 8, 70, 1024, 512, str(torch.bfloat16), True)
    assert key in tuning.TUNINGS and all(c["exact"] for c in tuning.TUNINGS[key]["candidates"])
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="warmed"):
        with torch.cuda.graph(graph):
            tuning.select(("never-seen",), lambda c: y0, [0], 0)


def test_one_call_grouped_linear_with_workspace():
    from actune_b200 import _lib, ops
    torch.manual_seed(4)
    x = torch.randn(33, 640, device="cuda", dtype=torch.bfloat16)
    codes, ws = ops.weight_codes((torch.randn(96, 640, device="cuda") * 0.02).bfloat16(), 2, 8)
    pw = ops.pack_rows(codes, 2)
    bias = torch.randn(96, device="cuda", dtype=torch.bfloat16)
    pa, as_ = ops.quantize_group64(x, 8)
    ref = ops.packed_linear(pa, as_, pw, ws, bias, 640, 2, 8)
    need = ops.workspace_size(33, 640, 8)
    assert need == 256 * ((33 * 640 + 255) // 256) + 256 * ((33 * 10 * 4 + 255) // 256)
    for _ in range(2):
        ws_buf = torch.full((need,), 0xAB, device="cuda", dtype=torch.uint8)
        y = ops.grouped_linear(x, pw, ws, bias, 2, 8, workspace=ws_buf)
        assert torch.equal(y, ref)
    with pytest.raises(_lib.ActuneError) as err:
        ops.grouped_linear(x, pw, ws, bias, 2, 8, workspace=torch.empty(need - 1, device="cuda", dtype=torch.uint8))
    assert err.value.status == _lib.ERR_WORKSPACE


def test_shared_activation_scope_reuses_quantization():
    from actune_b200.kernels import grouped as G
    torch.manual_seed(6)
    lin_a = torch.nn.Linear(256, 64, bias=False, device="cuda", dtype=torch.bfloat16)
    lin_b = torch.nn.Linear(256, 32, bias=False, device="cuda", dtype=torch.bfloat16)
    la, lb = G.GroupedLinear(lin_a, 4, 8, None), G.GroupedLinear(lin_b, 2, 8, None)
    x = torch.randn(12, 256, device="cuda", dtype=torch.bfloat16)
    ya, yb = la(x), lb(x)
    calls = []
    real = G.ops.quantize_group64

    def counting(*args, **kw):
        calls.append(1)
        return real(*args, **kw)

    G.ops.quantize_group64 = counting
    try:
        with G.shared_activation_scope(True):
            sa, sb = la(x), lb(x)
            x.add_(0)  # in-place update: the cached quantization must not be reused
            sc = la(x)
    finally:
        G.ops.quantize_group64 = real
    assert torch.equal(sa, ya) and torch.equal(sb, yb) and torch.equal(sc, ya)
    assert len(calls) == 2


@pytest.mark.parametrize("d", [256, 260, 4096, 8192])  # vectorised forms (D % 8 == 0) and the general one
def test_harness_glue_kernels(d):
    from actune_b200 import harness as H
    torch.manual_seed(8)
    x = torch.randn(7, d, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(7, d, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(d, device="cuda", dtype=torch.bfloat16)
    out, res = H.rmsnorm(x, w, 1e-5, r)
    s = (x.float() + r.float()).bfloat16().float()
    ref = w * (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-5)).bfloat16()
    assert torch.equal(res, s.bfloat16())
    assert float((out.float() - ref.float()).abs().max()) <= 2 ** -6 * float(ref.abs().max())
    inter = d // 2 + 4  # multiple of 8 only for some d
    gu = torch.randn(5, 2 * inter, device="cuda", dtype=torch.bfloat16)
    ga = H.gated_act(gu)
    g, u = gu.float().split(inter, -1)
    torch.testing.assert_close(ga.float(), (F.silu(g).bfloat16().float() * u), rtol=2e-2, atol=2e-2)
    for dh in (16, 128):
        qkv = torch.randn(6, (2 + 2 * 1) * dh, device="cuda", dtype=torch.bfloat16)
        cos, sin = H.rope_tables(6, dh, 10000.0, "cuda")
        before = qkv.clone()
        H.rope_(qkv, cos, sin, 2, 1, dh)
        q = before[:, :2 * dh].view(6, 2, dh).float()
        hd = dh // 2
        rot = torch.cat([q[..., :hd] * cos[:, None] - q[..., hd:] * sin[:, None],
                         q[..., hd:] * cos[:, None] + q[..., :hd] * sin[:, None]], -1)
        torch.testing.assert_close(qkv[:, :2 * dh].view(6, 2, dh).float(), rot, rtol=1e-2, atol=1e-2)
        assert torch.equal(qkv[:, 3 * dh:], before[:, 3 * dh:])  # v untouched


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_glue_kernels_quantize_like_the_quantizer(bits):
    """RMSNorm and the gated activation with the quantizing epilogue produce the
    bf16 output of the plain kernels and, bit for bit, the packed codes and scales
    of actune_quantize_group64 on that output."""
    import ctypes
    from actune_b200 import harness as H
    from actune_b200 import ops
    torch.manual_seed(bits)
    L = H._hlib()
    for d, gemma, with_res in ((256, False, True), (4096, False, False), (2048, True, True)):
        x = torch.randn(9, d, device="cuda", dtype=torch.bfloat16) * 3
        r = torch.randn(9, d, device="cuda", dtype=torch.bfloat16) if with_res else None
        w = torch.randn(d, device="cuda", dtype=torch.bfloat16)
        ref_out, ref_res = H.rmsnorm(x, w, 1e-5, r, gemma)
        for codes8 in (0, 1):
            width = 8 if codes8 else bits
            out = torch.empty_like(x)
            res_out = torch.empty_like(x) if with_res else None
            packed = torch.empty(9, d * width // 8, device="cuda", dtype=torch.uint8)
            scales = torch.empty(9, d // 64, device="cuda", dtype=torch.float32)
            rc = L.actune_harness_rmsnorm_q(H._p(x), H._p(r), H._p(w), H._p(out), H._p(res_out), 9, d,
                                            ctypes.c_float(1e-5), int(gemma), bits, codes8, H._p(packed),
                                            H._p(scales), H._s(x))
            assert rc == 0
            torch.cuda.synchronize()
            assert torch.equal(out, ref_out)
            if with_res:
                assert torch.equal(res_out, ref_res)
            qp, qs = ops.quantize_group64(out, bits, codes8=bool(codes8))
            assert torch.equal(packed, qp) and torch.equal(scales, qs)
    for inter, gelu in ((512, False), (11008, False), (1024, True)):
        gu = torch.randn(7, 2 * inter, device="cuda", dtype=torch.bfloat16)
        ref = H.gated_act(gu, gelu)
        for codes8 in (0, 1):
            width = 8 if codes8 else bits
            out = torch.empty_like(ref)
            packed = torch.empty(7, inter * width // 8, device="cuda", dtype=torch.uint8)
            scales = torch.empty(7, inter // 64, device="cuda", dtype=torch.float32)
            rc = L.actune_harness_gated_act_q(H._p(gu), H._p(out), 7, inter, int(gelu), bits, codes8, H._p(packed),
                                              H._p(scales), H._s(gu))
            assert rc == 0
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
            qp, qs = ops.quantize_group64(out, bits, codes8=bool(codes8))
            assert torch.equal(packed, qp) and torch.equal(scales, qs)


def test_small_oft_backbone_graph_vs_eager():
    """Graph replay (shared activation scope: the glue kernels hand the next
    projection its packed input) is bit-identical to eager calls (no scope: every
    projection quantizes its own input)."""
    from actune_b200.graph import GraphReplay
    from actune_b200.harness import OFTBackbone, build_w4a8_bank
    from actune_b200.layers import install_bank
    from actune_b200.precision import precision_profile
    model = OFTBackbone(layers=2, hidden=256, heads=4, mlp=512, tokens=40, action_tokens=8, chunk=(8,))
    bank, clips = build_w4a8_bank(model, 40)
    runtime = install_bank(model, bank, clips)
    x = torch.randn(40, 256, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        eager = {q: model(x).clone() for q in ("q00", "q11")}
    for q in ("q00", "q11"):
        with precision_profile(q), torch.inference_mode():
            eager[q] = model(x).clone()
    for shared in (False, True):
        policy = GraphReplay(model.forward, runtime.modules, shared_a8=shared)
        policy.enabled = True
        for q in ("q00", "q11", "q00"):
            with precision_profile(q), torch.inference_mode():
                assert torch.equal(policy(x), eager[q])
        policy.release()
    assert not torch.equal(eager["q00"], eager["q11"])


def test_graph_replay_literal_constants_and_shared_inputs():
    """Literal CUDA constants built inside the function are made while warming up and
    handed out as clones (the function may update them in place); graphs of several
    precisions for one input signature share one set of static inputs."""
    from actune_b200.graph import GraphReplay
    from actune_b200.layers import install_bank
    from actune_b200.precision import precision_profile
    model = tiny_model(2)
    runtime = install_bank(model, tiny_bank(model), {"0": {"w4a8": None, "w2a8": None},
                                                     "2": {"w4a8": None, "w2a8": None}})

    def step(x):
        t = torch.tensor(1.0, dtype=torch.float32, device="cuda")
        t += 0.5  # in place, as the reference's sampler updates its time tensor
        return model(x).float() * t

    x = torch.randn(4, 128, device="cuda", dtype=torch.bfloat16)
    with torch.inference_mode():
        eager = {q: None for q in ("q00", "q11")}
        for q in eager:
            with precision_profile(q):
                eager[q] = model(x).float() * 1.5
    replay = GraphReplay(step, runtime.modules)
    replay.enabled = True
    for q in ("q00", "q11", "q00", "q11"):
        with precision_profile(q), torch.inference_mode():
            out = replay(x.clone()).clone()
        assert torch.equal(out, eager[q]), q
    assert len(replay.graphs) == 2 and replay.replays == 4 and len(replay.constants) == 1
    assert len(replay._slots) == 1  # one static input set for both precisions
    replay.release()

    def late_literal(x):
        if torch.cuda.is_current_stream_capturing():
            torch.tensor(2.0, device="cuda")  # first seen during capture
        return x * 2

    late = GraphReplay(late_literal, {})
    late.enabled = True
    with pytest.raises(RuntimeError, match="Unwarmed CUDA constant"):
        late(torch.ones(3, device="cuda"))


def test_rope_cache_equals_rope_then_copy():
    """The rotary kernel that also writes the call's keys and values into a cache
    view whose sequences sit further apart than their length is bit-identical to the
    rotation followed by the copy."""
    from actune_b200 import harness as H
    heads, dh, batch, seq, offset, pitch = 8, 256, 3, 50, 304, 354
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = torch.randn(batch * seq, (heads + 2) * dh, device="cuda", generator=g).bfloat16()
    cos, sin = H.rope_tables(batch * seq, dh, 10000.0, "cuda")
    for view_len in (pitch, offset + seq):
        buf_a = torch.randn(batch, pitch, 2, dh, device="cuda", generator=g).bfloat16()
        buf_b = buf_a.clone()
        qa, qb = qkv.clone(), qkv.clone()
        H.rope_(qa, cos, sin, heads, 1, dh)
        buf_a[:, offset:offset + seq].copy_(qa[:, heads * dh:].view(batch, seq, 2, dh))
        H.rope_cache_(qb, cos, sin, heads, dh, buf_b[:, :view_len], seq, offset)
        assert torch.equal(qa, qb) and torch.equal(buf_a, buf_b)
