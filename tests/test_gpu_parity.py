"""GPU parity of every kernel against the CPU oracle and the reference goldens.

Tolerances (written per test):
  * fp32 outputs: relative error <= 1e-5 against the oracle / HF eager;
  * bf16 / fp16 outputs: <= 1 ULP against the oracle's reference algorithm
    (nearest-even store; the only differences come from the sum-of-squares
    order, exp and sin/cos), with >= 99.9 % of elements bit-identical;
    <= 1 ULP against the Triton-interpreter goldens (which truncate);
    <= 2 ULP against the eager PyTorch/HF compositions;
  * RoPE outputs: rotate-half is a difference of two products, so a 1-ULP
    difference in a normalised input or in a bf16 cos/sin value (sin/cos and
    the sum-of-squares order differ between CPU and GPU) can become several
    ULPs of a small, cancelled output.  An element passes when it is within
    1 ULP or within 2^-8 x the largest magnitude of its head vector (the size
    of such a one-ULP input change); at most 0.1 % of elements lie beyond
    2 ULP; >= 99 % of elements are bit-identical.  Given the kernel's own
    cos/sin and normed inputs the oracle reproduces its outputs bit for bit,
    and every element beyond 2 ULP is shown to sit on a differing input
    (test_rope_deviation_traces_to_cos_sin_and_norm_inputs);
  * KV-cache slots and V copies: bit-exact, and no other slot changes.
"""
from __future__ import annotations

import pytest
import torch

from golden_io import load
from oracle import kani_oracle as O

from kani_tts_b200 import StaticKVCache, fused_kernels as K, positions as P
from kani_tts_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def rnd(shape, seed, dtype=torch.bfloat16, mean=0.0, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (mean + std * torch.randn(shape, generator=g)).to(dtype)


def gpu(t):
    return t.to(DEV)


def ulp(a, b):
    return O.ulp_distance(a.cpu(), b.cpu())


def assert_close_ulp(got, ref, max_ulp=1, min_exact=0.999):
    d = ulp(got, ref)
    assert int(d.max()) <= max_ulp, f"max ULP {int(d.max())}"
    if d.numel():
        assert float((d == 0).float().mean()) >= min_exact, f"exact fraction {float((d == 0).float().mean())}"


def assert_rope_close(got, ref, min_exact=0.99, max_far_frac=1e-3):
    """RoPE outputs with in-kernel cos/sin against the oracle: every element within
    1 ULP, or within 2^-8 of its head's largest magnitude; at most `max_far_frac`
    of the elements beyond 2 ULP (each of those traces to a 1-ULP cos/sin or
    norm input: test_rope_deviation_traces_to_cos_sin_and_norm_inputs); at
    least `min_exact` bit-identical."""
    got, ref = got.cpu(), ref.cpu()
    d = ulp(got, ref)
    scale = ref.float().abs().amax(dim=-1, keepdim=True) * 2.0 ** -8
    ok = (d <= 1) | ((got.float() - ref.float()).abs() <= scale)
    far = int((d > 2).sum())
    assert bool(ok.all()), f"{int((~ok).sum())} elements outside tolerance, max ULP {int(d.max())}"
    if d.numel():
        assert far <= max_far_frac * d.numel(), f"{far} of {d.numel()} elements beyond 2 ULP"
        assert float((d == 0).float().mean()) >= min_exact, f"exact fraction {float((d == 0).float().mean())}"


def assert_attention_close(got, ref):
    """Attention output vs the float64 oracle: within 2 bf16 ULP, or within 2e-5
    absolute (outputs are weighted means of N(0, 1) values; where they cancel to
    ~1e-5, fp32 accumulation and the 2^-22 relative error of the hardware
    base-2 exponential are a few ULP of the tiny result); >= 95 % bit-identical."""
    got, ref = got.cpu(), ref.cpu()
    d = ulp(got, ref)
    ok = (d <= 2) | ((got.float() - ref.float()).abs() <= 2e-5)
    assert bool(ok.all()), f"{int((~ok).sum())} elements outside tolerance, max ULP {int(d.max())}"
    assert float((d == 0).float().mean()) >= 0.95


def assert_rel(got, ref, tol=1e-5):
    got, ref = got.cpu().float(), ref.cpu().float()
    rel = ((got - ref).abs() / ref.abs().clamp_min(1e-30))
    assert float(rel.max()) <= tol, float(rel.max())


@pytest.fixture(autouse=True)
def _clear_flags():
    _lib.read_and_clear_errors(DEV)
    yield


# ---------------------------------------------------------------- RMSNorm


@pytest.mark.parametrize("case", ["hidden_bf16", "decode_bf16", "qnorm_bf16", "knorm_bf16", "odd_bf16"])
def test_rms_norm_vs_reference_golden(case):
    c = load("triton_rms_norm")[case]
    y = K.fused_rms_norm(gpu(c["x"]), gpu(c["w"]), float(c["eps"]))
    assert y.shape == c["x"].shape and y.dtype == c["x"].dtype
    assert int(ulp(y, c["y"]).max()) <= 1                       # interpreter truncates
    assert_close_ulp(y, O.rms_norm_ref(c["x"], c["w"], float(c["eps"])))
    assert int(ulp(y, O.eager_rms_norm_hf(c["x"], c["w"], float(c["eps"]))).max()) <= 2


def test_rms_norm_fp32_is_true_fp32():
    c = load("triton_rms_norm")["fp32_storage"]
    y = K.fused_rms_norm(gpu(c["x"]), gpu(c["w"]), float(c["eps"]))
    assert y.dtype == torch.float32
    assert_rel(y, O.rms_norm_ref(c["x"], c["w"], float(c["eps"])), 1e-5)
    assert_rel(y, O.eager_rms_norm_hf(c["x"], c["w"], float(c["eps"])), 1e-5)
    assert not torch.equal(y.cpu(), y.cpu().to(torch.bfloat16).float())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [64, 100, 1024, 2048, 4096, 8192, 12000])
@pytest.mark.parametrize("rows", [1, 3, 257])
def test_rms_norm_shapes(dtype, n, rows):
    x = rnd((rows, n), 0, dtype)
    w = rnd((n,), 1, dtype, 1.0, 0.02)
    y = K.fused_rms_norm(gpu(x), gpu(w), 1e-5)
    ref = O.rms_norm_ref(x, w, 1e-5)
    if dtype == torch.float32:
        assert_rel(y, ref, 1e-5)
    else:
        assert_close_ulp(y, ref, 1, 0.995)


def test_rms_norm_mixed_weight_dtype_and_strided_rows():
    base = rnd((33, 1536), 2, torch.float32)
    x = gpu(base)[:, :1024]                       # row stride 1536: vector path with a stride
    w = rnd((1024,), 3, torch.bfloat16, 1.0, 0.02)
    y = K.fused_rms_norm(x, gpu(w), 1e-5)
    assert_rel(y, O.rms_norm_ref(base[:, :1024], w, 1e-5), 1e-5)


def test_rms_norm_misaligned_uses_generic_path():
    buf = gpu(rnd((5 * 1024 + 1,), 4))
    x = buf[1:].view(5, 1024)                    # 2-byte offset: not 16-byte aligned
    w = rnd((1024,), 5, torch.bfloat16, 1.0, 0.02)
    y = K.fused_rms_norm(x, gpu(w), 1e-5)
    assert_close_ulp(y, O.rms_norm_ref(x.cpu(), w, 1e-5))


# ------------------------------------------------------ residual + RMSNorm


def test_add_rms_norm_config1_fp32_vs_hf_golden():
    c = load("add_rms_norm")["config1_fp32_hf"]
    y, h = K.fused_add_rms_norm(gpu(c["x"]), gpu(c["r"]), gpu(c["w"]), float(c["eps"]))
    assert torch.equal(h.cpu(), c["h"])
    assert_rel(y, c["y"], 1e-5)


def test_add_rms_norm_bf16_vs_golden_and_in_place():
    c = load("add_rms_norm")["decode_bf16_triton"]
    x, r = gpu(c["x"]), gpu(c["r"])
    y, h = K.fused_add_rms_norm(x, r, gpu(c["w"]), float(c["eps"]))
    assert torch.equal(h.cpu(), c["h"])
    assert int(ulp(y, c["y"]).max()) <= 1
    yo, ho = O.add_rms_norm_ref(c["x"], c["r"], c["w"], float(c["eps"]))
    assert_close_ulp(y, yo)
    # in place: residual stream updated, normed output written over x
    K.fused_add_rms_norm(x, r, gpu(c["w"]), float(c["eps"]), out=x, residual_out=r)
    assert torch.equal(r.cpu(), ho) and torch.equal(x.cpu(), y.cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows", [1, 8, 1000, 16384])
def test_add_rms_norm_rows(dtype, rows):
    x, r = rnd((rows, 1024), 6, dtype), rnd((rows, 1024), 7, dtype)
    w = rnd((1024,), 8, dtype, 1.0, 0.02)
    y, h = K.fused_add_rms_norm(gpu(x), gpu(r), gpu(w), 1e-5)
    yo, ho = O.add_rms_norm_ref(x, r, w, 1e-5)
    assert torch.equal(h.cpu(), ho)
    if dtype == torch.float32:
        assert_rel(y, yo, 1e-5)
    else:
        assert_close_ulp(y, yo)


# ---------------------------------------------------------------- SiLU*mul


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("splits,rows,n", [(1, 1, 1024), (2, 64, 1024), (4, 64, 1024), (18, 5, 1024),
                                           (4, 300, 2048), (3, 7, 4096)])
def test_reduce_add_rms_norm_vs_oracle(dtype, splits, rows, n):
    """K-split fp32 partials summed in split order, rounded, added to the residual,
    RMSNorm: the residual sum bit-exact, the norm <= 1 ULP (fp32: 1e-5 relative)."""
    part = torch.randn(splits, rows, n, generator=torch.Generator().manual_seed(splits * 7 + rows)) * 0.3
    r = rnd((rows, n), 1310 + n, dtype)
    w = rnd((n,), 1311, dtype, 1.0, 0.02)
    y, h = K.reduce_add_rms_norm(gpu(part), gpu(r), gpu(w), 1e-5)
    yo, ho = O.reduce_add_rms_norm_ref(part, r, w, 1e-5)
    assert torch.equal(h.cpu(), ho)
    if dtype == torch.float32:
        assert_rel(y, yo, 1e-5)
    else:
        assert_close_ulp(y, yo)
    # row-major partials ([rows, splits, n] viewed as [splits, rows, n]) and in-place residual
    rm = gpu(part.transpose(0, 1).contiguous()).transpose(0, 1)
    rg = gpu(r)
    y2 = torch.empty_like(rg)
    K.reduce_add_rms_norm(rm, rg, gpu(w), 1e-5, out=y2, residual_out=rg)
    assert torch.equal(rg.cpu(), ho) and torch.equal(y2.cpu(), y.cpu())


def test_l2_prefetch_hint_on_norm_and_silu_changes_nothing():
    """reduce_add_rms_norm and fused_silu_mul with an L2 prefetch hint (a 20 MB
    weight buffer split over the launch's CTAs, in two ranges) give the same bytes
    as without one, and the hint is consumed by the call it was given to."""
    wbuf = torch.zeros(10 << 20, dtype=torch.bfloat16, device=DEV)
    half = wbuf.numel() // 2
    ranges = [(wbuf.data_ptr(), half * 2), (wbuf.data_ptr() + half * 2, half * 2)]
    part = gpu(torch.randn(6, 64, 1024, generator=torch.Generator().manual_seed(5)) * 0.3)
    r, w = gpu(rnd((64, 1024), 1330)), gpu(rnd((1024,), 1331, torch.bfloat16, 1.0, 0.02))
    y0, h0 = K.reduce_add_rms_norm(part, r, w, 1e-5)
    y1, h1 = K.reduce_add_rms_norm(part, r, w, 1e-5, l2_prefetch=ranges)
    assert torch.equal(y0, y1) and torch.equal(h0, h1)
    for t in (1, 64, 4096):
        gu = gpu(rnd((t, 2 * 4608), 1332 + t))
        a0 = K.fused_silu_mul(gu)
        a1 = K.fused_silu_mul(gu, l2_prefetch=ranges)
        assert torch.equal(a0, a1)
    torch.cuda.synchronize()
    assert _lib.read_and_clear_errors(DEV) == 0


def test_linear_split_k_sums_to_the_product():
    x = rnd((64, 4608), 1320)
    w = rnd((1024, 4608), 1321, std=0.03)
    p4 = K.linear_split_k(gpu(x), gpu(w), 4)
    assert p4.shape == (4, 64, 1024) and p4.dtype == torch.float32
    want = (x.double() @ w.double().t())
    assert float((p4.sum(0).double().cpu() - want).abs().max()) <= 1e-3 * float(want.abs().max())
    for s_ in range(4):                                   # each slice is the product over its K range
        sl = slice(s_ * 1152, (s_ + 1) * 1152)
        ws = x[:, sl].double() @ w[:, sl].double().t()
        assert float((p4[s_].double().cpu() - ws).abs().max()) <= 1e-3 * float(ws.abs().max())


@pytest.mark.parametrize("case", ["rows4_bf16", "decode_bf16", "odd_bf16"])
def test_silu_mul_vs_reference_golden(case):
    c = load("triton_silu_mul")[case]
    y = K.fused_silu_mul(gpu(c["gate_up"]))
    assert y.shape == c["y"].shape
    assert int(ulp(y, c["y"]).max()) <= 1
    assert_close_ulp(y, O.silu_mul_ref(c["gate_up"]))
    assert int(ulp(y, O.eager_silu_mul(c["gate_up"])).max()) <= 2


@pytest.mark.parametrize("t", [1, 64, 512, 4096, 32768])
def test_silu_mul_sweep(t):
    gu = rnd((t, 9216), 9)
    y = K.fused_silu_mul(gpu(gu))
    assert_close_ulp(y, O.silu_mul_ref(gu))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_silu_mul_other_dtypes(dtype):
    gu = rnd((17, 2 * 4608), 10, dtype)
    y = K.fused_silu_mul(gpu(gu))
    ref = O.silu_mul_ref(gu)
    if dtype == torch.float32:
        assert torch.allclose(y.cpu(), ref, rtol=1e-5, atol=1e-6)
    else:
        assert_close_ulp(y, ref)


@pytest.mark.parametrize("dtype,n", [(torch.bfloat16, 4608), (torch.float16, 4608), (torch.float32, 4608),
                                     (torch.bfloat16, 1000), (torch.bfloat16, 8192), (torch.float32, 6144)])
def test_silu_mul_row_per_cta_path(dtype, n):
    """Long calls (>= 2048 rows) take one CTA per row: every dtype, a width whose
    vectors do not fill the last 192-thread pass (n = 1000 bf16: 125 vectors),
    the widest row it takes (fp32 6144: 8 passes), a strided row view, and the
    extreme gate values of the short path."""
    rows = 2304
    gu = rnd((rows, 2 * n), 13, dtype)
    gu[0, :8] = torch.tensor([-100.0, -20.0, -1e-3, 0.0, 1e-3, 20.0, 88.0, -88.0], dtype=dtype)
    y = K.fused_silu_mul(gpu(gu))
    ref = O.silu_mul_ref(gu)
    if dtype == torch.float32:
        assert torch.allclose(y.cpu(), ref, rtol=1e-5, atol=1e-6)
    else:
        assert_close_ulp(y, ref)
    big = rnd((rows, 2 * n + 64), 14, dtype)
    ys = K.fused_silu_mul(gpu(big)[:, : 2 * n])
    refs = O.silu_mul_ref(big[:, : 2 * n])
    if dtype == torch.float32:
        assert torch.allclose(ys.cpu(), refs, rtol=1e-5, atol=1e-6)
    else:
        assert_close_ulp(ys, refs)


def test_silu_mul_strided_and_odd():
    big = rnd((9, 2 * 4608 + 64), 11)
    y = K.fused_silu_mul(gpu(big)[:, : 2 * 4608])          # row stride 9280, vector path
    assert_close_ulp(y, O.silu_mul_ref(big[:, : 2 * 4608]))
    odd = rnd((5, 2 * 77), 12)                               # n = 77: generic path
    assert_close_ulp(K.fused_silu_mul(gpu(odd)), O.silu_mul_ref(odd))


def test_silu_mul_extreme_values():
    g = torch.tensor([-100.0, -20.0, -1e-3, 0.0, 1e-3, 20.0, 88.0, -88.0])
    u = torch.ones_like(g) * 1.5
    gu = torch.cat([g, u]).reshape(1, 16).to(torch.bfloat16)
    y = K.fused_silu_mul(gpu(gu))
    assert_close_ulp(y, O.silu_mul_ref(gu), 1, 0.0)


# --------------------------------------------------------------- RoPE (ref)


@pytest.mark.parametrize("case", ["pos0", "pos1", "pos777", "pos2047"])
def test_rope_vs_reference_golden(case):
    c = load("triton_rope")[case]
    qo, ko = K.fused_rope(gpu(c["q"]), gpu(c["k"]), gpu(c["cos"]), gpu(c["sin"]))
    assert qo.shape == c["q"].shape and ko.shape == c["k"].shape
    assert int(ulp(qo, c["q_out"]).max()) <= 1 and int(ulp(ko, c["k_out"]).max()) <= 1
    # same fp32 operations, nearest-even store: bit-identical to the oracle
    assert torch.equal(qo.cpu(), O.rope_ref(c["q"], c["cos"], c["sin"]))
    assert torch.equal(ko.cpu(), O.rope_ref(c["k"], c["cos"], c["sin"]))


@pytest.mark.parametrize("d,dtype", [(32, torch.bfloat16), (128, torch.bfloat16), (64, torch.float32),
                                     (48, torch.bfloat16), (64, torch.float16)])
def test_rope_head_dims(d, dtype):
    q, k = rnd((1, 12, 1, d), 13, dtype), rnd((1, 4, 1, d), 14, dtype)
    cos, sin = rnd((d,), 15, dtype), rnd((d,), 16, dtype)    # arbitrary rows: halves differ
    qo, ko = K.fused_rope(gpu(q), gpu(k), gpu(cos), gpu(sin))
    assert torch.equal(qo.cpu(), O.rope_ref(q, cos, sin))
    assert torch.equal(ko.cpu(), O.rope_ref(k, cos, sin))


# ------------------------------------------------------------ KV write


@pytest.mark.parametrize("case", ["b1_slot5", "b2_slot0", "b1_last"])
def test_kv_cache_write_vs_static_cache_golden(case):
    c = load("static_cache_update")[case]
    kc, vc = gpu(c["k_prev"]), gpu(c["v_prev"])
    K.kv_cache_write(gpu(c["k"]), gpu(c["v"]), kc, vc, torch.tensor([int(c["slot"])], device=DEV))
    assert torch.equal(kc.cpu(), c["k_cache"]) and torch.equal(vc.cpu(), c["v_cache"])
    assert _lib.read_and_clear_errors(DEV) == 0


def test_kv_cache_write_per_stream_and_out_of_range():
    b = 4
    kc0, vc0 = rnd((b, 8, 16, 64), 17), rnd((b, 8, 16, 64), 18)
    k, v = rnd((b, 8, 1, 64), 19), rnd((b, 8, 1, 64), 20)
    slots = torch.tensor([3, 0, 15, 16])                      # last one out of range
    kc, vc = gpu(kc0), gpu(vc0)
    K.kv_cache_write(gpu(k), gpu(v), kc, vc, gpu(slots))
    ek, ev = kc0.clone(), vc0.clone()
    O.kv_write_ref(ek, ev, k, v, slots.tolist())
    assert torch.equal(kc.cpu(), ek) and torch.equal(vc.cpu(), ev)
    assert _lib.read_and_clear_errors(DEV) == _lib.KANI_FLAG_SLOT_OOB


def test_static_cache_update_matches_reference_semantics():
    class Cfg:
        num_key_value_heads, num_attention_heads, hidden_size = 8, 16, 1024
        num_hidden_layers, layer_types, conv_L_cache = 2, ["conv", "full_attention"], 3
    cache = StaticKVCache(Cfg, max_total_len=16, batch_size=2, device=DEV)
    k, v = rnd((2, 8, 1, 64), 21), rnd((2, 8, 1, 64), 22)
    cache.set_write_position(7)
    kf, vf = cache.update(gpu(k), gpu(v), 1)
    ek = torch.zeros(2, 8, 16, 64, dtype=torch.bfloat16)
    ev = ek.clone()
    O.kv_write_ref(ek, ev, k, v, 7)
    assert torch.equal(kf.cpu(), ek) and torch.equal(vf.cpu(), ev)
    assert cache.update(None, None, 0)[0].numel() == 0
    assert cache.read_errors() == 0


# ------------------------------------------------- fused RoPE + KV write


def _config2_case(seed, t=1, b=1, s_len=2048, p0=None, norm=False, table=True, dtype=torch.bfloat16,
                  hq=16, hk=8, d=64):
    g = torch.Generator().manual_seed(seed)
    n = b * t
    q = rnd((n, hq, d), seed + 1, dtype)
    k = rnd((n, hk, d), seed + 2, dtype)
    v = rnd((n, hk, d), seed + 3, dtype)
    inv = P.learnable_inv_freq(d, 1e6, 0.0)
    if p0 is None:
        pos = torch.randint(0, 2048, (n,), generator=g)
    else:
        pos = (p0 + torch.arange(t)).repeat(b)
    slots = pos.clone()
    tab = rnd((1024, d), seed + 4, dtype, 0.0, 0.02) if table else None
    qw = rnd((d,), seed + 5, dtype, 1.0, 0.02) if norm else None
    kw = rnd((d,), seed + 6, dtype, 1.0, 0.02) if norm else None
    kc = rnd((b, hk, s_len, d), seed + 7, dtype)
    vc = rnd((b, hk, s_len, d), seed + 8, dtype)
    return dict(q=q, k=k, v=v, inv=inv, pos=pos, slots=slots, tab=tab, qw=qw, kw=kw, kc=kc, vc=vc)


def _run_both(c, t, b, frame_pos=None, tpf=4):
    hq, d = c["q"].shape[1:]
    hk = c["k"].shape[1]
    kc, vc = gpu(c["kc"]), gpu(c["vc"])
    q_rot = K.fused_rope_kv_write(
        gpu(c["q"]).view(b, t, hq, d), gpu(c["k"]).view(b, t, hk, d), gpu(c["v"]).view(b, t, hk, d),
        gpu(c["inv"]), gpu(c["pos"]), kc, vc, gpu(c["slots"]),
        frame_table=None if c["tab"] is None else gpu(c["tab"]), tokens_per_frame=tpf,
        q_norm_w=None if c["qw"] is None else gpu(c["qw"]),
        k_norm_w=None if c["kw"] is None else gpu(c["kw"]), eps=1e-5,
        frame_pos=None if frame_pos is None else gpu(frame_pos))
    ekc, evc = c["kc"].clone(), c["vc"].clone()
    eq, flags = O.rope_kv_write_ref(c["q"], c["k"], c["v"], c["inv"], c["pos"], ekc, evc, c["slots"],
                                    frame_table=c["tab"], tokens_per_frame=tpf, q_norm_w=c["qw"],
                                    k_norm_w=c["kw"], eps=1e-5, frame_pos=frame_pos)
    return q_rot.reshape(eq.shape), kc, vc, eq, ekc, evc, flags


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
@pytest.mark.parametrize("norm", [False, True])
def test_rope_kv_write_config2_decode(seed, norm):
    c = _config2_case(100 + seed, norm=norm)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, 1, 1)
    assert flags == 0 and _lib.read_and_clear_errors(DEV) == 0
    assert_rope_close(q, eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)                       # V copy and untouched slots exact
    slot = int(c["slots"][0])
    mask = torch.ones(2048, dtype=torch.bool)
    mask[slot] = False
    assert torch.equal(kc.cpu()[:, :, mask], c["kc"][:, :, mask])


@pytest.mark.parametrize("t", [1, 64, 512, 4096])
def test_rope_kv_write_prefill_sweep(t):
    p0 = 0 if t == 4096 else 1000
    s_len = max(2048, p0 + t)
    c = _config2_case(200 + t, t=t, s_len=s_len, p0=p0, norm=True)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, t, 1)
    assert flags == 0 and _lib.read_and_clear_errors(DEV) == 0
    assert_rope_close(q, eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)


def test_rope_kv_write_batched_streams():
    b = 64
    c = _config2_case(300, t=1, b=b, norm=True)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, 1, b)
    assert flags == 0
    assert_rope_close(q, eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)


def test_rope_kv_write_packed_qkv_and_heads_major_output():
    b, t, hq, hk, d = 1, 37, 16, 8, 64
    c = _config2_case(400, t=t, b=b, p0=50, norm=True)
    qkv = torch.cat([c["q"].reshape(t, -1), c["k"].reshape(t, -1), c["v"].reshape(t, -1)], dim=1)
    qkv = gpu(qkv).view(b, t, (hq + 2 * hk) * d)
    q, k, v = qkv.split([hq * d, hk * d, hk * d], dim=-1)
    q_attn = torch.empty(b, hq, t, d, dtype=torch.bfloat16, device=DEV)   # SDPA layout
    kc, vc = gpu(c["kc"]), gpu(c["vc"])
    K.fused_rope_kv_write(q.view(b, t, hq, d), k.view(b, t, hk, d), v.view(b, t, hk, d), gpu(c["inv"]),
                          gpu(c["pos"]), kc, vc, gpu(c["slots"]), frame_table=gpu(c["tab"]),
                          q_norm_w=gpu(c["qw"]), k_norm_w=gpu(c["kw"]), q_out=q_attn.transpose(1, 2))
    ekc, evc = c["kc"].clone(), c["vc"].clone()
    eq, _ = O.rope_kv_write_ref(c["q"], c["k"], c["v"], c["inv"], c["pos"], ekc, evc, c["slots"],
                                frame_table=c["tab"], q_norm_w=c["qw"], k_norm_w=c["kw"])
    assert_rope_close(q_attn.transpose(1, 2).reshape(t, hq, d), eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)


def test_rope_kv_write_out_of_range_slot_and_frame():
    c = _config2_case(500, t=4, p0=0)
    c["slots"] = torch.tensor([0, 2048, -1, 5])             # two bad slots
    fp = torch.tensor([0, 4096, 8, -4])                      # frames 0, 1024 (bad), 2, -1 (bad)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, 4, 1, frame_pos=fp)
    assert flags == 3
    assert _lib.read_and_clear_errors(DEV) == 3
    assert_rope_close(q, eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)


@pytest.mark.parametrize("dtype,d,hq,hk", [(torch.float32, 64, 16, 8), (torch.float16, 64, 16, 8),
                                           (torch.bfloat16, 128, 8, 2), (torch.bfloat16, 48, 4, 2),
                                           (torch.bfloat16, 64, 48, 4), (torch.bfloat16, 32, 12, 12)])
def test_rope_kv_write_dtypes_and_generic_path(dtype, d, hq, hk):
    c = _config2_case(600, t=9, p0=100, norm=True, dtype=dtype, hq=hq, hk=hk, d=d)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, 9, 1)
    assert flags == 0
    if dtype == torch.float32:
        assert torch.allclose(q.cpu(), eq, rtol=1e-5, atol=1e-5)
        assert torch.allclose(kc.cpu(), ekc, rtol=1e-5, atol=1e-5)
    else:
        assert_rope_close(q, eq)
        assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)


def test_rope_kv_write_matches_reference_decode_composition():
    """Against the reference's decode sequence on the same inputs: per-head
    RMSNorm, cos/sin rows, RoPE and scatter_ (optimized_decode.py:220-240),
    each step through the oracle restatement of that step."""
    c = _config2_case(700, norm=True, table=False)
    pos = int(c["pos"][0])
    qn = O.rms_norm_ref(c["q"], c["qw"], 1e-5)
    kn = O.rms_norm_ref(c["k"], c["kw"], 1e-5)
    cos, sin = O.rope_cos_sin_ref(c["inv"], pos)
    q_ref, k_ref = O.rope_ref(qn, cos, sin), O.rope_ref(kn, cos, sin)
    q, kc, vc, *_ = _run_both(c, 1, 1)
    assert_rope_close(q, q_ref)
    assert_rope_close(kc.cpu()[0, :, pos], k_ref[0])
    assert torch.equal(vc.cpu()[0, :, pos], c["v"][0])


def test_update_fused_through_static_cache():
    class Cfg:
        num_key_value_heads, num_attention_heads, hidden_size = 8, 16, 1024
        num_hidden_layers, layer_types, conv_L_cache = 1, ["full_attention"], 3
    b = 3
    cache = StaticKVCache(Cfg, max_total_len=64, batch_size=b, device=DEV, per_stream_positions=True)
    c = _config2_case(800, t=1, b=b, s_len=64, norm=True, table=False)
    c["pos"] = torch.tensor([5, 9, 63])
    c["slots"] = c["pos"].clone()
    c["kc"] = torch.zeros(b, 8, 64, 64, dtype=torch.bfloat16)
    c["vc"] = torch.zeros_like(c["kc"])
    cache.set_write_position(gpu(c["slots"]))
    q_rot, kf, vf = cache.update_fused(gpu(c["q"]).view(b, 1, 16, 64), gpu(c["k"]).view(b, 1, 8, 64),
                                       gpu(c["v"]).view(b, 1, 8, 64), 0, gpu(c["inv"]),
                                       gpu(c["pos"]).view(b, 1), gpu(c["qw"]), gpu(c["kw"]))
    ekc, evc = c["kc"].clone(), c["vc"].clone()
    eq, _ = O.rope_kv_write_ref(c["q"], c["k"], c["v"], c["inv"], c["pos"], ekc, evc, c["slots"],
                                q_norm_w=c["qw"], k_norm_w=c["kw"])
    assert_rope_close(q_rot.reshape(eq.shape), eq)
    assert_rope_close(kf, ekc, 0.999)
    assert torch.equal(vf.cpu(), evc)


# ---------------------------------------------------------- graph capture


def test_ops_capture_in_cuda_graph():
    """Every op launches on the current stream without syncing: capture once,
    replay with new positions/slots written into the static inputs."""
    hq, hk, d, s_len = 16, 8, 64, 128
    c = _config2_case(900, t=1, s_len=s_len, norm=True)
    x, r = gpu(rnd((1, 1024), 901)), gpu(rnd((1, 1024), 902))
    w = gpu(rnd((1024,), 903, mean=1.0, std=0.02))
    gu = gpu(rnd((1, 9216), 904))
    q, k, v = gpu(c["q"]).view(1, 1, hq, d), gpu(c["k"]).view(1, 1, hk, d), gpu(c["v"]).view(1, 1, hk, d)
    kc, vc = gpu(c["kc"][:, :, :s_len]).contiguous(), gpu(c["vc"][:, :, :s_len]).contiguous()
    pos = torch.zeros(1, dtype=torch.long, device=DEV)
    slot = torch.zeros(1, dtype=torch.long, device=DEV)
    inv, tab, qw, kw = gpu(c["inv"]), gpu(c["tab"]), gpu(c["qw"]), gpu(c["kw"])
    _lib.error_flag(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):                               # warm-up outside capture
        K.fused_add_rms_norm(x, r, w, 1e-5)
        K.fused_silu_mul(gu)
        K.fused_rope_kv_write(q, k, v, inv, pos, kc, vc, slot, frame_table=tab, q_norm_w=qw, k_norm_w=kw)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y, h = K.fused_add_rms_norm(x, r, w, 1e-5)
        a = K.fused_silu_mul(gu)
        qo = K.fused_rope_kv_write(q, k, v, inv, pos, kc, vc, slot, frame_table=tab, q_norm_w=qw, k_norm_w=kw)
    for p in (5, 77, 127):
        pos.fill_(p)
        slot.fill_(p)
        g.replay()
        torch.cuda.synchronize()
        ekc, evc = c["kc"][:, :, :s_len].clone(), c["vc"][:, :, :s_len].clone()
        eq, _ = O.rope_kv_write_ref(c["q"], c["k"], c["v"], c["inv"], torch.tensor([p]), ekc, evc,
                                    torch.tensor([p]), frame_table=c["tab"], q_norm_w=c["qw"],
                                    k_norm_w=c["kw"])
        assert_rope_close(qo.reshape(eq.shape), eq)
        assert_rope_close(kc.cpu()[:, :, p], ekc[:, :, p])
    yo, ho = O.add_rms_norm_ref(x.cpu(), r.cpu(), w.cpu(), 1e-5)
    assert torch.equal(h.cpu(), ho)
    assert_close_ulp(y, yo)
    assert_close_ulp(a, O.silu_mul_ref(gu.cpu()))
    del g


def test_errors_raise_before_launch_on_gpu_tensors():
    x = gpu(rnd((2, 64), 1))
    with pytest.raises(TypeError):
        K.fused_rms_norm(x.to(torch.int32), gpu(rnd((64,), 2)))
    with pytest.raises(ValueError):
        K.fused_rms_norm(x, gpu(rnd((32,), 2)))
    with pytest.raises(ValueError):
        K.fused_silu_mul(gpu(rnd((2, 9), 3)))
    with pytest.raises(ValueError):
        K.fused_add_rms_norm(x, gpu(rnd((2, 32), 4)), gpu(rnd((64,), 2)))
    kc = torch.zeros(1, 8, 16, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        K.kv_cache_write(gpu(rnd((1, 8, 2, 64), 5)), gpu(rnd((1, 8, 1, 64), 5)), kc, kc.clone(),
                         torch.zeros(1, dtype=torch.long, device=DEV))


def test_rope_kv_write_bulk_partial_group_and_unaligned_metadata():
    """Long calls take the bulk-copy kernel: a token count that is not a
    multiple of its 4-token groups, and position/slot arrays that are not
    16-byte aligned (so they are loaded per warp instead of bulk-copied)."""
    t = 1030
    c = _config2_case(1000, t=t, s_len=2048, p0=17, norm=True)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, t, 1)
    assert flags == 0 and _lib.read_and_clear_errors(DEV) == 0
    assert_rope_close(q, eq)
    assert_rope_close(kc, ekc, 0.999)
    assert torch.equal(vc.cpu(), evc)
    # same call with the metadata arrays at an 8-byte offset
    pos_buf = torch.zeros(t + 1, dtype=torch.long, device=DEV)
    slot_buf = torch.zeros(t + 1, dtype=torch.long, device=DEV)
    pos_buf[1:] = gpu(c["pos"])
    slot_buf[1:] = gpu(c["slots"])
    kc2, vc2 = gpu(c["kc"]), gpu(c["vc"])
    q2 = K.fused_rope_kv_write(gpu(c["q"]).view(1, t, 16, 64), gpu(c["k"]).view(1, t, 8, 64),
                               gpu(c["v"]).view(1, t, 8, 64), gpu(c["inv"]), pos_buf[1:], kc2, vc2,
                               slot_buf[1:], frame_table=gpu(c["tab"]), q_norm_w=gpu(c["qw"]),
                               k_norm_w=gpu(c["kw"]))
    assert torch.equal(q2.cpu().reshape(q.shape), q.cpu())
    assert torch.equal(kc2.cpu(), kc.cpu()) and torch.equal(vc2.cpu(), vc.cpu())


def _kernel_cos_sin(inv, pos, d=64):
    """The kernel's own rounded cos/sin rows [N, D] at positions `pos` [N], read back
    through RoPE of the unit vector [1 ... 1 | 0 ... 0] (y = [cos | sin])."""
    n = pos.numel()
    x = torch.zeros(1, n, 1, d, dtype=torch.bfloat16, device=DEV)
    x[..., : d // 2] = 1.0
    kc = torch.zeros(1, 1, n, d, dtype=torch.bfloat16, device=DEV)
    y = K.fused_rope_kv_write(x, x.clone(), x.clone(), gpu(inv), gpu(pos), kc, torch.zeros_like(kc),
                              torch.arange(n, device=DEV)).reshape(n, d).cpu()
    c, s = y[:, : d // 2], y[:, d // 2:]
    return torch.cat([c, c], -1), torch.cat([s, s], -1)


def _kernel_norms(c, t, b):
    """The kernel's own q/k RMSNorm outputs: the same call at angle 0 (cos 1, sin 0:
    the rotation is the identity) without the frame table."""
    hq, d = c["q"].shape[1:]
    hk = c["k"].shape[1]
    n = b * t
    kc = torch.zeros(b, hk, t, d, dtype=torch.bfloat16, device=DEV)
    qn = K.fused_rope_kv_write(
        gpu(c["q"]).view(b, t, hq, d), gpu(c["k"]).view(b, t, hk, d), gpu(c["v"]).view(b, t, hk, d),
        gpu(c["inv"]), torch.zeros(n, dtype=torch.long, device=DEV), kc, torch.zeros_like(kc),
        torch.arange(t, device=DEV).repeat(b), q_norm_w=gpu(c["qw"]), k_norm_w=gpu(c["kw"]), eps=1e-5)
    return qn.reshape(n, hq, d).cpu(), kc.transpose(1, 2).reshape(n, hk, d).cpu()


@pytest.mark.parametrize("t,norm", [(1, False), (1, True), (64, False), (512, True), (4096, False),
                                    (4096, True)])
def test_rope_deviation_traces_to_cos_sin_and_norm_inputs(t, norm):
    """Accounting for every RoPE output element beyond 2 bf16 ULP of the oracle.

    1. Given the kernel's own rounded cos/sin rows and (with q/k norm) its own
       normed heads, the oracle's rotate-half + frame term + one rounding
       reproduces the kernel's Q output and K cache rows bit for bit: the
       rotation arithmetic is the reference's exactly.
    2. Those inputs are within 1 ULP of the oracle's (torch's cos/sin of the
       same fp32 angles; the oracle's norm).
    3. Every output element more than 2 ULP from the plain oracle sits on a
       lane whose own cos/sin value or one of whose two normed inputs (x_i,
       x_paired) differs from the oracle's: rotate-half subtracts two
       products, so a 1-ULP input change can move a cancelled output by many
       of its own ULPs.
    Config 2 shapes (Q 16 heads, K/V 8, D 64, theta 1e6, frame table [1024, 64]),
    decode (T = 1, p ~ U[0, 2047]) and the prefill sweep (consecutive p)."""
    b = 1
    p0 = None if t == 1 else (17 if t < 4096 else 0)      # frames p // 4 stay inside the 1024-row table
    c = _config2_case(2000 + t + (7 if norm else 0), t=t, s_len=max(2048, t + 17), p0=p0, norm=norm)
    q, kc, vc, eq, ekc, evc, flags = _run_both(c, t, b)
    assert flags == 0 and _lib.read_and_clear_errors(DEV) == 0
    n, d = b * t, 64
    slots = c["slots"]
    k_rows = kc.cpu()[0, :, slots].transpose(0, 1)          # [N, Hk, D]
    ek_rows = ekc[0, :, slots].transpose(0, 1)
    kcos, ksin = _kernel_cos_sin(c["inv"], c["pos"])
    ocos, osin = O.rope_cos_sin_ref(c["inv"], c["pos"])
    assert int(ulp(kcos, ocos).max()) <= 1 and int(ulp(ksin, osin).max()) <= 1
    if norm:
        qn, kn = _kernel_norms(c, t, b)
        oqn, okn = O.rms_norm_ref(c["q"], c["qw"], 1e-5), O.rms_norm_ref(c["k"], c["kw"], 1e-5)
        assert int(ulp(qn, oqn).max()) <= 1 and int(ulp(kn, okn).max()) <= 1
    else:
        qn, kn, oqn, okn = c["q"], c["k"], c["q"], c["k"]
    rows = c["tab"][torch.div(c["pos"], 4, rounding_mode="floor")]
    # 1. bit-exact given the kernel's own inputs
    assert torch.equal(q.cpu(), O.rope_compose_ref(qn, kcos, ksin, rows))
    assert torch.equal(k_rows, O.rope_compose_ref(kn, kcos, ksin, rows))
    assert torch.equal(vc.cpu(), evc)
    # 3. every element beyond 2 ULP of the oracle traces to a differing input
    half = d // 2
    stats = {}
    for name, got, want, xk, xo in (("q", q.cpu(), eq, qn, oqn), ("k", k_rows, ek_rows, kn, okn)):
        dist = ulp(got, want)
        far = dist > 2
        cs_diff = ((kcos != ocos) | (ksin != osin)).unsqueeze(1)                  # [N, 1, D]
        x_diff = xk != xo
        pair_diff = torch.cat([x_diff[..., half:], x_diff[..., :half]], -1)
        explained = cs_diff | x_diff | pair_diff
        assert bool((~far | explained).all()), f"{name}: {int((far & ~explained).sum())} unexplained elements"
        stats[name] = (int(far.sum()), far.numel(), int(dist.max()))
    print(f"rope T={t} norm={norm}: elements > 2 ULP of the oracle (all traced to a 1-ULP cos/sin or norm "
          f"input): Q {stats['q'][0]}/{stats['q'][1]} (max {stats['q'][2]} ULP), "
          f"K {stats['k'][0]}/{stats['k'][1]} (max {stats['k'][2]} ULP)")


@pytest.mark.parametrize("t", [64, 65536])
def test_in_kernel_cos_sin_match_cuda_math(t):
    """The kernel's shared-reduction sin/cos, read back through RoPE of a unit
    vector (x = [1 ... 1 | 0 ... 0] gives y = [cos | sin]), against CUDA's own
    cosf/sinf (torch on the GPU) of the same fp32 angles, both rounded to
    bf16: at most 1 ULP apart and almost always identical."""
    d = 64
    inv = gpu(P.learnable_inv_freq(d, 1e6, 0.0))
    pos = torch.arange(t, dtype=torch.long, device=DEV)
    q = torch.zeros(1, t, 1, d, dtype=torch.bfloat16, device=DEV)
    q[..., : d // 2] = 1.0
    k, v = q.clone(), q.clone()
    kc = torch.zeros(1, 1, t, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    y = K.fused_rope_kv_write(q, k, v, inv, pos, kc, vc, pos).reshape(t, d)
    ang = inv[None, :] * pos.float()[:, None]            # fp32 angles, as the reference forms them
    ref_c, ref_s = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    for got, ref in ((y[:, : d // 2], ref_c), (y[:, d // 2:], ref_s)):
        dist = ulp(got, ref)
        assert int(dist.max()) <= 1
        assert float((dist != 0).float().mean()) < 1e-4


# ------------------------------------------------ decode attention / short conv


@pytest.mark.parametrize("b,hq,hk,s_len,lens", [(1, 16, 8, 2048, [1629]), (3, 16, 8, 512, [1, 7, 512]),
                                                (2, 8, 8, 64, [33, 64]), (2, 16, 4, 300, [250, 9]),
                                                # enough streams that the split drops to 2 and 1 CTAs
                                                # (the largest split whose grid is one wave)
                                                (24, 16, 8, 256, [(37 * i) % 256 + 1 for i in range(24)]),
                                                (40, 16, 8, 256, [(37 * i) % 256 + 1 for i in range(40)]),
                                                (80, 16, 8, 256, [(53 * i) % 256 + 1 for i in range(80)])])
def test_decode_attention_vs_oracle(b, hq, hk, s_len, lens):
    d = 64
    q = rnd((b, hq, d), 1100)
    kc, vc = rnd((b, hk, s_len, d), 1101), rnd((b, hk, s_len, d), 1102)
    kv_len = torch.tensor(lens, dtype=torch.long)
    got = K.decode_attention(gpu(q), gpu(kc), gpu(vc), gpu(kv_len))
    ref = O.decode_attention_ref(q, kc, vc, kv_len, d ** -0.5)
    assert_attention_close(got, ref)
    assert _lib.read_and_clear_errors(DEV) == 0


def test_decode_attention_ignores_slots_past_the_prefix_and_flags_overflow():
    b, hq, hk, s_len, d = 2, 16, 8, 128, 64
    q = rnd((b, hq, d), 1110)
    kc, vc = rnd((b, hk, s_len, d), 1111), rnd((b, hk, s_len, d), 1112)
    kv_len = torch.tensor([40, 128])
    got = K.decode_attention(gpu(q), gpu(kc), gpu(vc), gpu(kv_len))
    kc2, vc2 = kc.clone(), vc.clone()
    kc2[0, :, 40:] = 1e4                           # garbage beyond the prefix must not matter
    vc2[0, :, 40:] = -1e4
    got2 = K.decode_attention(gpu(q), gpu(kc2), gpu(vc2), gpu(kv_len))
    assert torch.equal(got.cpu(), got2.cpu())
    K.decode_attention(gpu(q), gpu(kc), gpu(vc), gpu(torch.tensor([40, 129])))
    assert _lib.read_and_clear_errors(DEV) == _lib.KANI_FLAG_SLOT_OOB


@pytest.mark.parametrize("b,lens", [(1, [100]), (1, [1629]), (3, [5, 640, 1200]), (4, [2048, 1, 64, 65])])
def test_decode_attention_step_after_the_kv_write(b, lens):
    """kani_decode_attention_step launched right behind the fused QKV GEMV +
    RoPE + KV write, which releases its dependents early and writes q and each
    stream's newest row (kv_len - 1): bit-identical to kani_decode_attention,
    eagerly and replayed from a CUDA graph, and close to the oracle.  The newest
    row falls in a first-stage tile (100 slots over 8 CTAs) and in a later one
    (1629 slots)."""
    hq, hk, d, h, s_len = 16, 8, 64, 1024, 2048
    kv_len = torch.tensor(lens, dtype=torch.long)
    slots = kv_len - 1
    x = gpu(rnd((b, 1, h), 1130))
    res = gpu(rnd((b, 1, h), 1131))
    nw = gpu((1.0 + 0.1 * rnd((h,), 1132, torch.float32)).to(torch.bfloat16))
    w = gpu(rnd(((hq + 2 * hk) * d, h), 1133, std=0.03))
    inv = gpu(P.learnable_inv_freq(d, 1e6, 0.0))
    kc0, vc0 = rnd((b, hk, s_len, d), 1134), rnd((b, hk, s_len, d), 1135)
    pos, sl, kl = gpu(slots), gpu(slots), gpu(kv_len)

    def chain(prefix_final, kc, vc, hbuf, out):
        q_rot = K.gemv_rope_kv_write(x, w, nw, inv, pos, kc, vc, sl, num_q_heads=hq, num_kv_heads=hk,
                                     residual=res, residual_out=hbuf)
        return K.decode_attention(q_rot, kc, vc, kl, out=out, prefix_final=prefix_final)

    runs = {}
    for mode in (False, True):
        kc, vc = gpu(kc0), gpu(vc0)
        hbuf = torch.empty_like(x)
        out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=DEV)
        chain(mode, kc, vc, hbuf, out)
        torch.cuda.synchronize()
        runs[mode] = (out.clone(), kc.clone(), vc.clone())
        # the same chain captured and replayed (the rows it writes are rewritten identically)
        s = torch.cuda.Stream(device=DEV)
        s.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(s):
            chain(mode, kc, vc, hbuf, out)
        torch.cuda.current_stream(DEV).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            chain(mode, kc, vc, hbuf, out)
        out.zero_()
        g.replay()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, runs[mode][0])
    assert torch.equal(runs[True][0], runs[False][0])
    q_rot = K.gemv_rope_kv_write(x, w, nw, inv, pos, gpu(kc0), gpu(vc0), sl, num_q_heads=hq, num_kv_heads=hk,
                                 residual=res, residual_out=torch.empty_like(x))
    ref = O.decode_attention_ref(q_rot.reshape(b, hq, d).cpu(), runs[True][1].cpu(), runs[True][2].cpu(), kv_len,
                                 d ** -0.5)
    assert_attention_close(runs[True][0], ref)
    assert _lib.read_and_clear_errors(DEV) == 0


def _lens(b: int, seed: int) -> list[int]:
    """Valid lengths for b streams: the newest row in a first-stage tile (100
    slots), in a later tile (1629), at both ends (1, 2048), and seeded others."""
    fixed = [100, 1629, 1, 2048, 65]
    g = torch.Generator().manual_seed(seed)
    extra = torch.randint(1, 2049, (max(0, b - len(fixed)),), generator=g).tolist()
    return (fixed + extra)[:b]


@pytest.mark.parametrize("b", [5, 8, 64])
def test_decode_attention_step_after_the_token_rope_kv_write(b):
    """kani_decode_attention_step behind the token-kernel RoPE + KV write
    (fused_rope_kv_write with q/k norm on packed QKV views, the producer of the
    5-64-stream decode paths), which releases its dependents at entry and
    writes q and each stream's newest row: bit-identical to
    kani_decode_attention, eagerly and replayed from a CUDA graph, and close to
    the oracle.  Each stream's newest row first holds other values, so a read
    of the stale row would change the output."""
    hq, hk, d, s_len = 16, 8, 64, 2048
    kv_len = torch.tensor(_lens(b, 1140 + b), dtype=torch.long)
    slots = kv_len - 1
    qkv = gpu(rnd((b, 1, (hq + 2 * hk) * d), 1141))
    qv = qkv[..., :hq * d].view(b, 1, hq, d)
    kv = qkv[..., hq * d:(hq + hk) * d].view(b, 1, hk, d)
    vv = qkv[..., (hq + hk) * d:].view(b, 1, hk, d)
    qw = gpu((1.0 + 0.1 * rnd((d,), 1142, torch.float32)).to(torch.bfloat16))
    kw = gpu((1.0 + 0.1 * rnd((d,), 1143, torch.float32)).to(torch.bfloat16))
    inv = gpu(P.learnable_inv_freq(d, 1e6, 0.0))
    kc0, vc0 = rnd((b, hk, s_len, d), 1144), rnd((b, hk, s_len, d), 1145)
    pos, sl, kl = gpu(slots // 4 + 3), gpu(slots), gpu(kv_len)

    def chain(prefix_final, kc, vc, out):
        q_rot = K.fused_rope_kv_write(qv, kv, vv, inv, pos, kc, vc, sl, q_norm_w=qw, k_norm_w=kw, eps=1e-5)
        return K.decode_attention(q_rot, kc, vc, kl, out=out, prefix_final=prefix_final)

    runs = {}
    for mode in (False, True):
        kc, vc = gpu(kc0), gpu(vc0)
        out = torch.empty(b, hq, d, dtype=torch.bfloat16, device=DEV)
        chain(mode, kc, vc, out)
        torch.cuda.synchronize()
        runs[mode] = (out.clone(), kc.clone(), vc.clone())
        # captured and replayed from a fresh cache copy: the stale rows are back in place
        kc.copy_(gpu(kc0))
        vc.copy_(gpu(vc0))
        s = torch.cuda.Stream(device=DEV)
        s.wait_stream(torch.cuda.current_stream(DEV))
        with torch.cuda.stream(s):
            chain(mode, kc, vc, out)
        torch.cuda.current_stream(DEV).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            chain(mode, kc, vc, out)
        for _ in range(3):
            kc.copy_(gpu(kc0))
            vc.copy_(gpu(vc0))
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, runs[mode][0])
            assert torch.equal(kc, runs[mode][1]) and torch.equal(vc, runs[mode][2])
    assert torch.equal(runs[True][0], runs[False][0])
    for i in range(b):   # the newest rows were rewritten
        assert not torch.equal(runs[True][1][i, :, int(slots[i])].cpu(), kc0[i, :, int(slots[i])])
    q_rot = K.fused_rope_kv_write(qv, kv, vv, inv, pos, gpu(kc0), gpu(vc0), sl, q_norm_w=qw, k_norm_w=kw, eps=1e-5)
    ref = O.decode_attention_ref(q_rot.reshape(b, hq, d).cpu(), runs[True][1].cpu(), runs[True][2].cpu(), kv_len,
                                 d ** -0.5)
    assert_attention_close(runs[True][0], ref)
    assert _lib.read_and_clear_errors(DEV) == 0


@pytest.mark.parametrize("b,h", [(1, 1024), (64, 1024), (3, 256)])
def test_short_conv_step_bit_exact_vs_eager(b, h):
    bcx = rnd((b, 3 * h), 1200)
    state = rnd((b, h, 3), 1201)
    w = rnd((h, 3), 1202, std=0.3)
    st_gpu = gpu(state)
    y = K.short_conv_step(gpu(bcx), st_gpu, gpu(w))
    st_ref = state.clone()
    y_ref = O.short_conv_step_ref(bcx, st_ref, w)
    assert torch.equal(st_gpu.cpu(), st_ref)
    assert int(ulp(y, y_ref).max()) <= 1            # three-term fp32 sum order
    assert float((ulp(y, y_ref) == 0).float().mean()) > 0.999


def test_decode_attention_strided_cache_uses_register_path():
    """A [B, S, Hk, D] cache viewed as [B, Hk, S, D] (slot stride != head_dim)
    takes the register kernel; same results as the oracle."""
    b, hq, hk, s_len, d = 2, 16, 8, 300, 64
    q = rnd((b, hq, d), 1120)
    kc_bshd, vc_bshd = rnd((b, s_len, hk, d), 1121), rnd((b, s_len, hk, d), 1122)
    kc, vc = gpu(kc_bshd).permute(0, 2, 1, 3), gpu(vc_bshd).permute(0, 2, 1, 3)
    kv_len = torch.tensor([300, 77])
    got = K.decode_attention(gpu(q), kc, vc, gpu(kv_len))
    ref = O.decode_attention_ref(q, kc_bshd.permute(0, 2, 1, 3), vc_bshd.permute(0, 2, 1, 3), kv_len, d ** -0.5)
    assert_attention_close(got, ref)
