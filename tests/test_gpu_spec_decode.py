"""The speculative decode loop (``specverify.draft.spec_decode``) on a tiny
random-init Llama-shaped model: with greedy acceptance, speculative decoding
must produce exactly the target's own greedy continuation -- the defining
property of the reference's loop (``diffspec_model.py:268-754``).  The plain
continuation is decoded one token at a time through the same model (one-row
verify steps); a step fed the true continuation as a chain must accept all of
it, and the compacted cache must then continue the same sequence."""
from __future__ import annotations

import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

PROMPT = 300


def _model():
    from specverify.draft.spec_decode import LlamaShape, SpecDecodeModel
    shape = LlamaShape(hidden=512, layers=4, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1000,
                       draft_vocab=1000, feature_layers=(0, 1, 2))
    m = SpecDecodeModel.from_config(shape, device="cuda", seed=0, max_tokens=1024, draft_ctx=256)
    # well-separated logits: the argmax cannot flip on rounding differences
    # between a 1-row and a many-row step
    m.lm_head.normal_(0.0, 1.0, generator=torch.Generator(device="cuda").manual_seed(9))
    return m


def _plain_greedy(m, root: int, start: int, n: int):
    """Target greedy decode, one token per step through the same kernels."""
    from specverify.runtime import pack_tree_mask
    bits = pack_tree_mask(torch.ones(1, 1, dtype=torch.int8, device="cuda"))[0]
    out = []
    tok = root
    for i in range(n):
        ids = torch.tensor([tok], device="cuda")
        pos = torch.tensor([start + i], device="cuda")
        hidden, _ = m.verify(ids, pos, bits, start + i)
        tok = int(torch.argmax((hidden @ m.lm_head.t()).float(), dim=-1).item())
        out.append(tok)
    return out


def test_greedy_speculative_decode_equals_target_greedy():
    m = _model()
    root = m.fill_context(PROMPT, seed=4)
    want = _plain_greedy(m, root, PROMPT, 24)
    r = m.diffspec_generate(PROMPT, max_new_tokens=24, nodes=8, max_depth=4, temperature=0.0, seed=4)
    assert r["tokens"] == want
    assert r["final_length"] == PROMPT + sum(a + 1 for a in r["accepted_per_step"])


def test_chain_of_the_true_continuation_is_fully_accepted_and_compacted():
    from specverify.runtime.draft_tree import finalize_tree
    m = _model()
    root = m.fill_context(PROMPT, seed=5)
    want = _plain_greedy(m, root, PROMPT, 12)
    depth = 5
    # a width-1 tree: root -> want[0] -> ... -> want[depth-1]
    tree = finalize_tree(torch.arange(depth, device="cuda"), torch.zeros(depth, 1, dtype=torch.int64, device="cuda"),
                         torch.tensor(want[:depth], device="cuda").view(depth, 1), depth, 1, validate=True)
    root_t = torch.tensor([root], device="cuda")
    feat = torch.zeros(1, 3 * m.shape.hidden, device="cuda", dtype=m.dtype)
    m.fill_context(PROMPT, seed=5)                      # the plain decode wrote past the prompt: restore
    acc, _, _ = m.step(root_t, feat, PROMPT, 1, depth, 0.0, 0, 0, tree=tree)
    h = acc.to_host()
    assert h["accept_length"] == depth
    assert h["best_candidate"][1:] == want[:depth]
    assert h["next_token"] == want[depth]
    # the compacted cache continues the same greedy sequence
    rest = _plain_greedy(m, want[depth], PROMPT + depth + 1, 12 - depth - 1)
    assert rest == want[depth + 1:12]


def test_graphed_verify_equals_eager_verify():
    """The verify step replayed from per-layer-boundary CUDA graphs computes
    what the eager forward does, on the same cache state, for two successive
    steps (the second reuses the captured graphs at another cache length)."""
    from specverify.runtime import pack_tree_mask
    m = _model()
    m.fill_context(PROMPT, seed=6)
    t = 9
    keep = torch.tril(torch.ones(t, t, dtype=torch.int8, device="cuda"))
    bits = pack_tree_mask(keep)[0]                      # [M, words]
    g = torch.Generator(device="cuda").manual_seed(1)
    for start in (PROMPT, PROMPT + 5):
        ids = torch.randint(0, m.shape.vocab, (t,), device="cuda", generator=g)
        pos = start + torch.arange(t, device="cuda")
        h_e, f_e = m.verify(ids, pos, bits, start)
        h_e, f_e = h_e.clone(), f_e.clone()
        h_g, f_g = m.verify_graphed(ids, pos, bits, start)
        torch.cuda.synchronize()
        assert torch.allclose(h_g.float(), h_e.float(), atol=1e-2, rtol=1e-2)
        assert torch.allclose(f_g.float(), f_e.float(), atol=1e-2, rtol=1e-2)
        assert (h_g != h_e).float().mean().item() < 1e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_rms_norm_and_silu_mul_match_the_reference_formulas(dtype):
    """tv_rms_norm / tv_silu_mul against LlamaRMSNorm and SiLU(gate) * up as
    the reference writes them in torch: equal up to one rounding of the
    output type (the fp32 sum of squares is accumulated in another order)."""
    from specverify.draft.spec_decode import rms_norm, silu_mul
    g = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(65, 4096, device="cuda", generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(4096, device="cuda", generator=g)).to(dtype)
    xf = x.float()
    want = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(dtype) * w
    got = rms_norm(x, w, 1e-5)
    assert torch.allclose(got.float(), want.float(), rtol=1 / 64, atol=1e-6)
    assert (got != want).float().mean().item() < 0.01
    # a row-strided view (every other row) and an offset weight slice
    w2 = torch.cat([w, w])
    got2 = rms_norm(x[::2], w2[4096:], 1e-5)
    assert torch.equal(got2, got[::2])
    gu = (torch.randn(65, 2 * 1024, device="cuda", generator=g) * 4).to(dtype)
    want = torch.nn.functional.silu(gu[:, :1024]) * gu[:, 1024:]
    got = silu_mul(gu, 1024)
    assert torch.allclose(got.float(), want.float(), rtol=1 / 64, atol=1e-6)
    assert (got != want).float().mean().item() < 0.001
