"""Generate the fused decode+unpack golden vectors (unpack_*.npz) by running the reference's own
GPU kernel.

The reference's fused Gated DeltaNet decode (ConvUpdateUnpack, causal_conv1d_cute/unpack.py:33-222,
called through causal_conv1d_update_unpack, unpack.py:328-374) has no CPU path, so these vectors
come from its CuTe kernel on a B200. Run on a GPU machine where the reference package is
installed (for instance under baseline/_ref, where bench.py's reference arm looks for it):

    python tests/golden/make_golden_unpack.py [--ref baseline/_ref] [--out tests/golden]

The reference needs nvidia-cutlass-dsl >= 4.6, whose cute.math.tanh takes `approx=`; with 4.5.0
(the version in this image) the same function spells it `fastmath=`. The only change made here is
that keyword forwarding, applied to the DSL before the reference is imported; the reference's
sources are run as they are. Inputs are seeded on the CPU and copied to the GPU. Every case runs
the public entry point with the launch shape the reference picks itself (unpack_config). Stored:
inputs, outputs (conv output, Z, B, A) and the state cache after the call. Rows whose slot is the
pad id or outside the cache get their conv input as output and keep their state.
The tests never import the reference; they read only the .npz files.
"""

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

# (name, B, D, zdim, heads, W, dtype, gdtype, slots, extra row columns, bias, activation)
CASES = [
    ("unpack_0_bf16_w4", 8, 256, 64, 16, 4, torch.bfloat16, torch.bfloat16, 16, 0, True, "silu"),
    ("unpack_1_f16_w2", 5, 512, 128, 8, 2, torch.float16, torch.float16, 9, 0, False, None),
    ("unpack_2_bf16_w8_gf32", 33, 512, 256, 32, 8, torch.bfloat16, torch.float32, 36, 0, True, "silu"),
    ("unpack_3_bf16_w3_rows", 6, 512, 512, 16, 3, torch.bfloat16, torch.bfloat16, 8, 8, False, "silu"),
    ("unpack_4_f32_w5", 4, 128, 32, 4, 5, torch.float32, torch.float32, 6, 0, True, "silu"),
    ("unpack_5_bf16_w4_b64", 64, 1024, 512, 32, 4, torch.bfloat16, torch.bfloat16, 66, 0, True, "silu"),
]
PAD = -1


def _install_compat():
    import cutlass.cute as cute

    tanh = cute.math.tanh

    def tanh_compat(a, fastmath=False, *, approx=None, **kw):
        return tanh(a, fastmath or bool(approx), **kw)

    cute.math.tanh = tanh_compat


def _store(d, name, t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        d[name + "@bf16"] = t.view(torch.int16).numpy().view(np.uint16)
    elif t.dtype == torch.float16:
        d[name + "@f16"] = t.numpy()
    elif t.dtype == torch.float32:
        d[name + "@f32"] = t.numpy()
    else:
        d[name + "@" + str(t.dtype).replace("torch.", "")] = t.numpy()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--ref", default=str(ROOT / "baseline" / "_ref"))
    p.add_argument("--out", default=str(HERE))
    args = p.parse_args()
    sys.path.insert(0, args.ref)
    _install_compat()
    import causal_conv1d_cute as R
    from causal_conv1d_cute import fallback, unpack

    assert Path(R.__file__).resolve().is_relative_to(Path(args.ref).resolve()), R.__file__

    def refuse(why):
        raise RuntimeError(f"reference would fall back to PyTorch: {why}")

    fallback.warn = refuse
    out_dir = Path(args.out)
    out_dir.mkdir(parents=True, exist_ok=True)
    dev = torch.device("cuda", 0)
    for seed, (name, B, D, zdim, heads, W, dt, gdt, slots, extra, has_bias, act) in enumerate(CASES):
        g = torch.Generator().manual_seed(100 + seed)
        qkvz_wide = torch.randn(B, D + zdim + extra, generator=g).to(dt)
        ba = torch.randn(B, 2 * heads, generator=g).to(gdt)
        w = ((torch.rand(D, W, generator=g) - 0.5)).to(dt)
        bias = (torch.randn(D, generator=g) * 0.1).to(dt) if has_bias else None
        st0 = torch.randn(slots, D, W - 1, generator=g).to(dt)
        idx = torch.randperm(slots, generator=g)[:B].to(torch.int32)
        idx[0] = PAD
        if B > 3:
            idx[3] = slots + 7  # outside the cache: the reference skips it like a pad row
        qd = qkvz_wide.to(dev)[:, : D + zdim]
        bad, std = ba.to(dev), st0.to(dev)
        wd = w.to(dev)
        bd = None if bias is None else bias.to(dev)
        reason = unpack.unpack_reason(qd, bad, std, wd, bd, heads)
        assert reason is None, (name, reason)
        vec, bs = unpack.unpack_config(D, B, qd.stride(0))
        o, z, b, a = unpack.causal_conv1d_update_unpack(qd, bad, std, wd, bd, idx.to(dev), heads,
                                                        act, PAD, vec, bs)
        torch.cuda.synchronize()
        meta = {"B": B, "D": D, "zdim": zdim, "heads": heads, "W": W, "slots": slots,
                "row_extra": extra, "act": act, "pad": PAD, "vec": vec, "bs": bs,
                "source": "reference ConvUpdateUnpack (CuTe DSL) on B200"}
        d = {"meta": np.array(json.dumps(meta))}
        for k, v in dict(qkvz=qkvz_wide[:, : D + zdim], ba=ba, w=w, state0=st0, out=o, z=z,
                         b=b, a=a, state=std).items():
            _store(d, k, v)
        if bias is not None:
            _store(d, "bias", bias)
        d["idx@int32"] = idx.numpy()
        np.savez_compressed(out_dir / f"{name}.npz", **d)
        print(name, "vec", vec, "bs", bs, flush=True)


if __name__ == "__main__":
    main()
