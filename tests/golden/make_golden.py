"""Generate the golden vectors in this directory by running the reference implementation.

Run once, in a checkout that has the reference package importable (its CPU path, the PyTorch
fallback, needs no GPU):

    PYTHONPATH=<path to causal-conv1d-cute> python tests/golden/make_golden.py

Every case calls the reference's public API (causal_conv1d_fn, causal_conv1d_varlen_fn,
causal_conv1d_update, causal_conv1d_update_ring, to_ring, from_ring) with CPU tensors, which the
reference serves with causal_conv1d_cute/fallback.py, and stores inputs and outputs in one .npz
per case. bf16 tensors are stored as their raw uint16 bit patterns (key suffix "@bf16"). Outputs
that the reference leaves undefined (rows skipped as padding) are listed in a mask.
The tests never import the reference; they read only these files.
"""

import json
import warnings
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _store(d, name, t):
    if t is None:
        return
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        d[name + "@bf16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float16:
        d[name + "@f16"] = t.numpy()
    elif t.dtype == torch.float32:
        d[name + "@f32"] = t.numpy()
    elif t.dtype == torch.bool:
        d[name + "@bool"] = t.numpy()
    else:
        d[name + "@" + str(t.dtype).replace("torch.", "")] = t.numpy()


def _save(name, meta, **tensors):
    d = {"meta": np.array(json.dumps(meta))}
    for k, v in tensors.items():
        _store(d, k, v)
    np.savez_compressed(HERE / f"{name}.npz", **d)


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _u(shape, g, dtype, lo=-0.5, hi=0.5):
    return (torch.rand(shape, generator=g) * (hi - lo) + lo).to(dtype)


def fn_cases(C):
    # BASELINE config 1 exactly: x (2,256,512) fp32 N(0,1), w U(-.5,.5), b N(0,.1), silu.
    g = _gen(1)
    x = torch.randn(2, 256, 512, generator=g)
    w = _u((256, 4), g, torch.float32)
    b = torch.randn(256, generator=g) * 0.1
    y = C.causal_conv1d_fn(x, w, b, "silu")
    _save("fn_config1", {"op": "fn", "act": "silu", "layout": "bdl"}, x=x, w=w, b=b, out=y)
    # Widths, bias, activation and both layouts in bf16 / fp16 at small sizes.
    i = 0
    for W in (2, 3, 4, 5, 8):
        for dtype, layout, act, has_bias in (
            (torch.bfloat16, "btd", "silu", True),
            (torch.bfloat16, "bdl", None, False),
            (torch.float16, "btd", "silu", False),
        ):
            g = _gen(100 + i)
            i += 1
            B, D, L = 2, 64, 37
            if layout == "btd":
                x = torch.randn(B, L, D, generator=g).to(dtype).transpose(1, 2)
            else:
                x = torch.randn(B, D, L, generator=g).to(dtype)
            w = _u((D, W), g, dtype)
            b = (torch.randn(D, generator=g) * 0.1).to(dtype) if has_bias else None
            y = C.causal_conv1d_fn(x, w, b, act)
            _save(f"fn_w{W}_{layout}_{str(dtype)[6:]}", {"op": "fn", "act": act, "layout": layout},
                  x=x.contiguous(), w=w, b=b, out=y.contiguous())


def varlen_cases(C):
    PAD = -1
    cases = [
        # (W, lens, pads, with_states, extra_rows)
        (4, [5, 1, 30, 2, 3, 4, 17], [0, 0, 1, 0, 0, 0, 0], True, 0),
        (2, [1, 2, 9, 0, 40], [0, 0, 0, 0, 0], True, 3),
        (3, [2, 2, 3, 1, 25], [0, 1, 0, 0, 0], True, 0),
        (8, [3, 7, 8, 1, 20, 33], [0, 0, 0, 0, 0, 1], True, 5),
        (4, [6, 11, 1], [0, 0, 0], False, 0),
    ]
    for n, (W, lens, pads, with_states, extra) in enumerate(cases):
        g = _gen(200 + n)
        D, K = 32, W - 1
        nseq = len(lens)
        slots = nseq + 3
        qsl = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
        T = int(qsl[-1]) + extra
        perm = torch.randperm(slots, generator=g)[:nseq].to(torch.int32)
        cidx = perm.clone()
        cidx[torch.tensor(pads, dtype=torch.bool)] = PAD
        hinit = torch.rand(nseq, generator=g) < 0.5
        x = torch.randn(T, D, generator=g).to(torch.bfloat16).t()  # token-major view
        w = _u((D, W), g, torch.bfloat16)
        b = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16) if n % 2 == 0 else None
        st0 = torch.randn(slots, D, K, generator=g).to(torch.bfloat16)
        st = st0.clone() if with_states else None
        y = C.causal_conv1d_varlen_fn(x, w, b, qsl, cidx if with_states else None,
                                      hinit if with_states else None, st, "silu", PAD)
        mask = torch.zeros(D, T, dtype=torch.bool)  # defined outputs
        for i in range(nseq):
            a, e = int(qsl[i]), int(qsl[i + 1])
            if not (with_states and pads[i]):
                mask[:, a:e] = True
        _save(f"varlen_{n}_w{W}", {"op": "varlen", "act": "silu", "pad": PAD, "states": with_states},
              x=x.contiguous(), w=w, b=b, qsl=qsl, cidx=cidx, hinit=hinit, st0=st0,
              st=st, out=y.contiguous(), mask=mask)


def update_cases(C):
    PAD = -1
    # (name, W, B, L, D, state_len, inter_layout, indexed, pads, dtype)
    cases = [
        ("single_idx", 4, 6, 1, 48, 3, None, True, [0, 0, 1, 0, 0, 0], torch.bfloat16),
        ("single_direct", 3, 4, 1, 32, 2, None, False, [0, 0, 0, 0], torch.float32),
        ("multi_dense", 4, 5, 3, 32, 3, "dense", True, [0, 1, 0, 0, 0], torch.bfloat16),
        ("multi_dedup", 3, 4, 4, 32, 2, "dedup", True, [0, 0, 0, 1], torch.bfloat16),
        ("multi_none", 5, 3, 5, 16, 4, None, True, [0, 0, 0], torch.float16),
        ("long_state_w3", 3, 4, 1, 32, 4, None, False, [0, 0, 0, 0], torch.bfloat16),
        ("long_state_w4", 4, 3, 2, 16, 6, None, True, [0, 0, 0], torch.bfloat16),
        ("single_w8", 8, 3, 1, 16, 7, "dense", True, [0, 0, 0], torch.bfloat16),
    ]
    for n, (name, W, B, L, D, S, layout, indexed, pads, dtype) in enumerate(cases):
        g = _gen(300 + n)
        K = W - 1
        slots = B + 4 if indexed else B
        xs = torch.randn(B, L, D, generator=g).to(dtype).transpose(1, 2)  # (B, D, L) view
        x = xs[..., 0].contiguous() if L == 1 and layout is None else xs
        w = _u((D, W), g, dtype)
        b = (torch.randn(D, generator=g) * 0.1).to(dtype) if n % 2 == 0 else None
        st0 = torch.randn(slots, D, S, generator=g).to(dtype)
        idx = iidx = None
        if indexed:
            idx = torch.randperm(slots, generator=g)[:B].to(torch.int32)
            idx[torch.tensor(pads, dtype=torch.bool)] = PAD
            iidx = torch.randperm(slots, generator=g)[:B].to(torch.int32)
        phys = inter = None
        if layout == "dense":
            phys = torch.full((slots, L, D, K), 7.0).to(dtype)
            inter = phys
        elif layout == "dedup":
            PW = L + K - 1
            phys = torch.full((slots, D, PW), 7.0).to(dtype)
            inter = phys.as_strided((slots, L, D, K), (D * PW, 1, PW, 1))
        st = st0.clone()
        ph0 = None if phys is None else phys.clone()
        y = C.causal_conv1d_update(x, st, w, b, "silu" if n % 3 != 1 else None, idx, PAD,
                                   inter, iidx if inter is not None else None)
        mask = torch.tensor([not p for p in pads])
        _save(f"update_{name}", {"op": "update", "act": "silu" if n % 3 != 1 else None, "pad": PAD,
                                 "inter": layout, "L": L},
              x=x.contiguous(), w=w, b=b, st0=st0, st=st, idx=idx, iidx=iidx,
              inter0=ph0, inter=None if phys is None else phys, out=y.contiguous(), mask=mask)


def ring_cases(C):
    PAD = -1
    for n, (W, B, D, indexed, dtype) in enumerate([(4, 5, 32, True, torch.bfloat16),
                                                   (3, 3, 16, False, torch.float32),
                                                   (8, 4, 16, True, torch.bfloat16)]):
        g = _gen(400 + n)
        K = W - 1
        slots = B + 3 if indexed else B
        ordered = torch.randn(slots, D, K, generator=g).to(dtype)
        seen = torch.randint(0, 97, (slots,), generator=g, dtype=torch.int32)
        ring0 = C.to_ring(ordered, seen).contiguous()
        w = _u((D, W), g, dtype)
        b = (torch.randn(D, generator=g) * 0.1).to(dtype)
        idx = None
        rows = torch.arange(B)
        if indexed:
            idx = torch.randperm(slots, generator=g)[:B].to(torch.int32)
            idx[1] = PAD
            rows = idx.long()
        ring = ring0.clone()
        steps = {}
        lens_all = seen.clone()
        for s in range(3):
            x = torch.randn(B, D, generator=g).to(dtype)
            lens = lens_all[rows.clamp_min(0)] if indexed else lens_all.clone()
            y = C.causal_conv1d_update_ring(x, ring, w, b, "silu", lens, idx, PAD)
            steps[f"x{s}"] = x
            steps[f"lens{s}"] = lens.clone()
            steps[f"out{s}"] = y
            steps[f"ring_after{s}"] = ring.clone()
            live = rows[rows >= 0] if indexed else rows
            lens_all[live] += 1
        mask = torch.tensor([True] * B)
        if indexed:
            mask[1] = False
        _save(f"ring_{n}_w{W}", {"op": "ring", "act": "silu", "pad": PAD, "steps": 3},
              ring0=ring0, w=w, b=b, idx=idx, mask=mask, **steps)
    g = _gen(450)
    st = torch.randn(7, 32, 3, generator=g)
    seen = torch.randint(0, 50, (7,), generator=g, dtype=torch.int32)
    r = C.to_ring(st, seen)
    _save("ring_convert", {"op": "convert"}, state=st, seen=seen, ring=r.contiguous(),
          back=C.from_ring(r, seen))


def main():
    import causal_conv1d_cute as C

    warnings.simplefilter("ignore")
    torch.manual_seed(0)
    fn_cases(C)
    varlen_cases(C)
    update_cases(C)
    ring_cases(C)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
