"""The torch.library ops (wfd::attn, wfd::wave_attn, wfd::commit, ...) without a
GPU: schemas with their declared mutations, fake (meta) kernels that give the
output shapes under FakeTensorMode, and no CPU kernel (a CPU call fails in the
dispatcher instead of computing somewhere else)."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import __graft_entry__

__graft_entry__.load_package()
from wavefront_decoding_b200 import ops  # noqa: E402,F401  (registers torch.ops.wfd.*)


def test_schemas_declare_mutations():
    s = str(torch.ops.wfd.wave_attn.default._schema)
    assert "Tensor(a!) k_cache" in s and "Tensor(b!) v_cache" in s and "Tensor(c!)? lens" in s
    assert "Tensor q," in s and "Tensor items" in s  # inputs that are only read
    s = str(torch.ops.wfd.commit.default._schema)
    assert "Tensor(a!) k_cache" in s and "Tensor(c!) lens" in s and s.endswith("-> (Tensor, Tensor)")
    assert "Tensor(a!) lens" in str(torch.ops.wfd.commit_drop.default._schema)
    s = str(torch.ops.wfd.attn.default._schema)
    assert "!" not in s and s.endswith("-> Tensor")
    assert "Tensor(a!) out" in str(torch.ops.wfd.attn_out.default._schema)


def test_fake_kernels_give_shapes():
    with FakeTensorMode():
        q = torch.empty(64, 16, 128, dtype=torch.bfloat16)
        kn = torch.empty(64, 4, 128, dtype=torch.bfloat16)
        kc = torch.empty(8, 8, 4096, 4, 128, dtype=torch.bfloat16)
        items = torch.empty(64, 5, dtype=torch.int32)
        lens = torch.empty(8, 8, dtype=torch.int32)
        out = torch.ops.wfd.wave_attn(q, kn, kn, kc, kc.clone(), items, 1, lens, 0, None, -1)
        assert out.shape == q.shape and out.dtype == q.dtype
        cu = torch.empty(65, dtype=torch.int32)
        out = torch.ops.wfd.attn(q, kn, kn, cu, cu, 1, 4096, True, None)
        assert out.shape == q.shape
        rows, cnt = torch.ops.wfd.commit(kc, kc.clone(), lens, items, torch.empty(64, dtype=torch.int32), None, 0, 512)
        assert rows.shape == (512,) and cnt.shape == (64,) and rows.dtype == torch.int32


def test_no_cpu_kernel():
    q = torch.zeros(2, 4, 64)
    k = torch.zeros(5, 4, 64)
    cu = torch.tensor([0, 2], dtype=torch.int32)
    cuk = torch.tensor([0, 5], dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        torch.ops.wfd.attn(q, k, k, cu, cuk, 2, 5, False, None)
