"""The tcgen05 prompt kernel (wfd_attn_prefill, K7) against the float64 oracle of
the reference's attn_dense (fa4_attention.py:191-232, _attn_dense_sdpa
:218-232): causal (bottom-right) and non-causal, MHA and GQA, head_dim 64 and
128, prompt lengths that are and are not multiples of the 128-row tile, and the
config-4 prompt length (1024) on the config-4 head shape.  bf16, max-abs 2e-2."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attention as oattn

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2

CASES = [
    # (name, B, Tq, Tk, H, Hkv, Dh, causal)
    ("mha_d64_causal_ragged", 2, 300, 300, 8, 8, 64, True),
    ("gqa4_d128_causal", 2, 257, 257, 16, 4, 128, True),
    ("mha_d64_noncausal", 2, 200, 200, 4, 4, 64, False),
    ("gqa2_d64_bottom_right", 3, 130, 333, 8, 4, 64, True),
    ("mha_d128_one_tile", 1, 128, 128, 2, 2, 128, True),
    ("cfg4_prompt_d64", 1, 1024, 1024, 24, 24, 64, True),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_prefill_kernel_vs_oracle(cuda_dev, case):
    from wavefront_decoding_b200 import attention as wa
    from wavefront_decoding_b200 import runtime as rt
    name, B, Tq, Tk, H, Hkv, Dh, causal = case
    g = gi.gen(sum(map(ord, name)))
    q = gi.randn((B, Tq, H, Dh), g, torch.bfloat16)
    k = gi.randn((B, Tk, Hkv, Dh), g, torch.bfloat16)
    v = gi.randn((B, Tk, Hkv, Dh), g, torch.bfloat16)
    out = wa.attn_prefill(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), causal=causal)
    torch.cuda.synchronize()
    assert rt.read_device_error(cuda_dev) == 0
    ref = oattn.attn_dense(q, k, v, causal=causal)
    err = float(np.abs(out.float().cpu().numpy() - ref).max())
    assert err < TOL_BF16, err
    # attn_dense (the reference surface) takes the same kernel for bf16 prompts
    out2 = wa.attn_dense(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), causal=causal)
    assert torch.equal(out2, out)


def test_prefill_kernel_repeatable_and_rows_without_keys(cuda_dev):
    """Identical launches give identical bits; with Tq > Tk (bottom-right
    causal) the first Tq - Tk rows see no key and come out as zeros, as in the
    oracle."""
    from wavefront_decoding_b200 import attention as wa
    g = gi.gen(5)
    B, Tq, Tk, H, Dh = 2, 200, 150, 4, 64
    q = gi.randn((B, Tq, H, Dh), g, torch.bfloat16).to(cuda_dev)
    k = gi.randn((B, Tk, H, Dh), g, torch.bfloat16).to(cuda_dev)
    v = gi.randn((B, Tk, H, Dh), g, torch.bfloat16).to(cuda_dev)
    a = wa.attn_prefill(q, k, v, causal=True)
    b = wa.attn_prefill(q, k, v, causal=True)
    assert torch.equal(a, b)
    assert float(a[:, :Tq - Tk].abs().max()) == 0.0
    ref = oattn.attn_dense(q.cpu(), k.cpu(), v.cpu(), causal=True)
    assert float(np.abs(a.float().cpu().numpy()[:, Tq - Tk:] - ref[:, Tq - Tk:]).max()) < TOL_BF16
