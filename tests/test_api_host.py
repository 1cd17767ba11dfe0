"""Host-side behaviour that needs no GPU: argument validation (same ValueError cases as the
reference), the no-fallback rule (unsupported calls raise), layout classification, the rebinding
helper, the accuracy classifier, and the shims' serve / pass-on decisions."""

import sys
import types

import pytest
import torch
import torch.nn.functional as F

import causal_conv1d_cute as C
from causal_conv1d_cute import _patch, dao_compat, functional as fn, sglang_compat
from causal_conv1d_cute import testing as T


def test_bad_shapes_raise_value_error():
    """Reference tests/test_fallback.py:85-97."""
    x = torch.randn(1, 64, 32, dtype=torch.bfloat16)
    w = torch.randn(48, 4, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        C.causal_conv1d_fn(x, w)
    with pytest.raises(ValueError):
        C.causal_conv1d_fn(x, torch.randn(64, 4, 2, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        C.causal_conv1d_update(x[:, :, 0], torch.zeros(1, 64, 1, dtype=torch.bfloat16),
                               torch.randn(64, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        C.causal_conv1d_varlen_fn(x[0], torch.randn(64, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        C.causal_conv1d_update_ring(x[:, :, 0], torch.zeros(1, 64, 3), torch.randn(64, 4))
    with pytest.raises(ValueError):
        C.causal_conv1d_fn(x, torch.randn(64, 4, dtype=torch.bfloat16), activation="relu")


def test_no_cpu_fallback():
    x = torch.randn(1, 32, 20)
    w = torch.randn(32, 4)
    assert not C.supported(x, w)
    with pytest.raises(C.Unsupported, match="not a CUDA tensor"):
        C.causal_conv1d_fn(x, w, None, "silu")
    with pytest.raises(C.Unsupported):
        C.causal_conv1d_update(x[:, :, 0], torch.zeros(3, 32, 3), w)
    qsl = torch.tensor([0, 20], dtype=torch.int32)
    with pytest.raises(C.Unsupported):
        C.causal_conv1d_varlen_fn(x[0], w, None, qsl)
    with pytest.raises(C.Unsupported):
        C.causal_conv1d_update_ring(x[:, :, 0], torch.zeros(1, 3, 32), w, None, None,
                                    torch.zeros(1, dtype=torch.int32))


def test_reasons():
    x = torch.randn(1, 32, 20, requires_grad=True)
    w = torch.randn(32, 4)
    assert "gradients" in fn._reason(x, w)
    with torch.no_grad():
        assert "CUDA" in fn._reason(x, w)
    assert "int32" in fn.varlen_reason(x[0].detach(), w, None, torch.tensor([0, 20]), None)
    assert fn.varlen_reason(x[0].detach(), w, None, None, None)
    assert fn._act(True) == "silu" and fn._act("swish") == "silu" and fn._act(False) is None


def test_inter_layout():
    S, L, D, K = 3, 4, 16, 3
    dense = torch.zeros(S, L, D, K)
    PW = L + K - 1
    dedup = torch.zeros(S, D, PW).as_strided((S, L, D, K), (D * PW, 1, PW, 1))
    assert fn._inter_layout(dense, D, K + 1, L, torch.float32) == "dense"
    assert fn._inter_layout(dedup, D, K + 1, L, torch.float32) == "dedup"
    assert fn._inter_layout(dense.transpose(2, 3), D, K + 1, L, torch.float32) is None
    assert fn._inter_layout(dense, D, K + 1, L + 1, torch.float32) is None


def test_in_place_prefill_refused_before_launch():
    x = torch.randn(1, 64, 16)
    w = torch.randn(64, 4)
    with pytest.raises(ValueError):
        C.CausalConv1d(w, None, None).fwd(x, out=x)
    with pytest.raises(ValueError):
        C.CausalConv1d(w, None, "relu")
    with pytest.raises(ValueError):
        C.CausalConv1d(torch.randn(64, 9), None, None)


def test_wrap_rebinds_every_importer_and_is_idempotent():
    """Reference tests/test_patch.py:15-37."""
    src = types.ModuleType("cc1d_fake_src")

    def f(a):
        return a + 1

    src.f = f
    user = types.ModuleType("cc1d_fake_user")
    user.g = f
    sys.modules["cc1d_fake_src"] = src
    sys.modules["cc1d_fake_user"] = user
    try:
        n = _patch.wrap("cc1d_fake_src.f", lambda orig, a: orig(a) * 10)
        assert n == 2
        assert src.f(1) == 20 and user.g(1) == 20
        assert src.f.__name__ == "f"
        assert _patch.wrap("cc1d_fake_src.f", lambda orig, a: 0) == 0
        assert user.g(2) == 30
    finally:
        del sys.modules["cc1d_fake_src"], sys.modules["cc1d_fake_user"]


@pytest.mark.parametrize(
    "D,W,act,bias", [(1536, 7, None, True), (2048, 3, None, False), (1024, 4, "silu", True)]
)
def test_check_classifies_known_outputs(D, W, act, bias):
    """Reference tests/test_accuracy_check.py:7-34, on the CPU."""
    case = T.Case("check", "fwd", D, W, 2, 512, bias, act, "bdl")
    t = T.make_inputs(case, device="cpu")
    ref = T.reference(case, t)
    x, w, b = t["x"], t["w"], t["b"]
    fin = (lambda y: F.silu(y)) if act else (lambda y: y)
    xp = F.pad(x, (W - 1, 0))
    acc = b.view(1, D, 1).expand(2, D, 512).clone() if bias else torch.zeros_like(x)
    for k in range(W):
        acc = acc + w[:, k].view(1, D, 1) * xp[..., k : k + 512]
    w_drop = w.clone()
    w_drop[:, 0] = 0
    dropped = fin(F.conv1d(x.float(), w_drop.float().unsqueeze(1), b.float() if bias else None,
                           padding=W - 1, groups=D)[..., :512]).to(case.dtype)
    assert T.check(case, t, ref.to(case.dtype), ref)[0] == "ok"
    assert T.check(case, t, fin(acc), ref)[0] == "lowprec"
    assert T.check(case, t, dropped, ref)[0] == "WRONG"
    assert T.check(case, t, torch.roll(ref.to(case.dtype), 1, dims=-1), ref)[0] == "WRONG"


def test_dao_shim_passes_unservable_calls_upstream():
    calls = []

    def upstream_fn(x, weight, bias=None, **kw):
        calls.append(kw)
        return "upstream"

    x = torch.randn(1, 32, 20)
    w = torch.randn(32, 4)
    before = dict(dao_compat.stats)
    assert dao_compat.around_fn(upstream_fn, x, w, None, seq_idx=torch.zeros(1)) == "upstream"
    assert dao_compat.around_fn(upstream_fn, x, w, None, activation="silu") == "upstream"  # CPU
    assert dao_compat.stats["fn_fallback"] == before["fn_fallback"] + 2

    def upstream_update(x, conv_state, weight, bias=None, **kw):
        return "upstream"

    assert dao_compat.around_update(upstream_update, x[:, :, 0], torch.zeros(1, 32, 3), w,
                                    cache_seqlens=torch.zeros(1)) == "upstream"


def test_sglang_shim_selection_and_pass_on(monkeypatch):
    monkeypatch.setenv(sglang_compat.ENV_PATHS, "fn")
    pairs = sglang_compat._wrappers()
    assert [t for t, _ in pairs] == list(sglang_compat.TARGETS_FN)
    monkeypatch.setenv(sglang_compat.ENV_PATHS, "fn,update,unpack")
    names = [t for t, _ in sglang_compat._wrappers()]
    assert set(sglang_compat.TARGETS_UPDATE) <= set(names)

    def original(*a, **k):
        return "original"

    x = torch.randn(32, 10)  # fewer than MIN_PREFILL_TOKENS tokens
    w = torch.randn(32, 4)
    qsl = torch.tensor([0, 10], dtype=torch.int32)
    assert sglang_compat.around_fn(original, x, w, None, query_start_loc=qsl) == "original"
    assert sglang_compat.around_update(original, x[:, 0].unsqueeze(0), torch.zeros(1, 32, 3), w,
                                       None, None, num_accept_tokens=torch.ones(1)) == "original"
    monkeypatch.setenv(sglang_compat.ENV_DRY_RUN, "1")
    assert sglang_compat._dry_run()
    assert sglang_compat.stats["fn_fallback"] >= 1
