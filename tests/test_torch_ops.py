"""The entry points are torch.library ops (cc1d::*) whose schemas mark the arguments each one
writes (outputs and caches), with fake implementations so that meta and fake tensors trace through
them without touching the GPU. The public functions call these ops; the GPU tests exercise them
with real data."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import causal_conv1d_cute  # noqa: F401  (registers the ops)

# op -> the argument names its schema marks as written
MUTATED = {
    "fwd": {"out"},
    "fwd_states": {"out", "final_states"},
    "update": {"state", "out3", "inter"},
    "update_ring": {"ring", "out"},
    "to_ring": {"ring"},
    "from_ring": {"state"},
    "varlen": {"out", "states"},
    "update_unpack": {"state", "out", "z", "b", "a"},
}


@pytest.mark.parametrize("name", sorted(MUTATED))
def test_op_is_registered_with_its_mutations(name):
    schema = getattr(torch.ops.cc1d, name).default._schema
    written = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
    assert written == MUTATED[name]
    assert len(schema.returns) == 0


def test_fake_and_meta_tensors_trace_without_the_gpu():
    bf = torch.bfloat16
    x = torch.empty(2, 64, 32, device="meta", dtype=bf)
    w = torch.empty(64, 4, device="meta", dtype=bf)
    assert torch.ops.cc1d.fwd(x, w, None, True, torch.empty_like(x)) is None
    with FakeTensorMode():
        xv = torch.empty(64, 100, dtype=bf)
        qsl = torch.tensor([0, 40, 100], dtype=torch.int32)
        st = torch.empty(4, 64, 3, dtype=bf)
        out = torch.empty_like(xv)
        wf = torch.empty(64, 4, dtype=bf)
        assert torch.ops.cc1d.varlen(xv, wf, None, True, out, qsl, None, None, st, -1) is None
