"""pkv_lm_head_argmax (the LM head fused with greedy selection) on the GPU.

The token ids are checked against the oracle (``oracle/lm_head.py``, pinned to the
reference's ``compute_logits`` + greedy ``Sampler`` in ``tests/golden``) and against the
reference's path run by torch on the same device (``F.linear(hidden, weight).float()``
then ``argmax``). Ids must be equal wherever the row's two best exact logits are more
than one model-dtype ulp apart (any float32-accumulated GEMM agrees there); on the rare
near-tie rows either leader is accepted. The largest logit must equal the oracle's
rounded one to within one ulp.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import lm_head as oracle

pytestmark = pytest.mark.gpu

NP_DTYPE = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from mini_inference_b200 import ops as _ops
    return _ops


def _case(vocab, hidden, batch, dtype, dev, seed, weight_std=0.02):
    g = torch.Generator(device="cpu").manual_seed(seed)
    w = (torch.randn(vocab, hidden, generator=g) * weight_std).to(dtype).to(dev)
    h = torch.randn(batch, hidden, generator=g).to(dtype).to(dev)
    return h, w


def _exact(h, w):
    """The oracle's exact logits, over vocabulary slices (bounded host memory at 7B sizes)."""
    hn = h.float().cpu().numpy()
    wc = w.cpu()
    return np.concatenate([oracle.exact_logits(hn, wc[i:i + 16384].float().numpy())
                           for i in range(0, wc.shape[0], 16384)], axis=1)


def _check(ids, top, h, w, dtype):
    name = NP_DTYPE[dtype]
    exact = _exact(h, w)
    ids = ids.cpu().numpy()
    want, want_top = oracle.greedy_from_exact(exact, name)
    amb = oracle.ambiguous_rows(exact, name)
    assert oracle.acceptable(exact, name, ids).all()
    np.testing.assert_array_equal(ids[~amb], want[~amb])
    if top is not None:
        top = top.cpu().numpy().astype(np.float64)
        assert (np.abs(top - want_top) <= oracle.ulp(want_top, name)).all()
    return amb


SHAPES = [  # (vocab, hidden, batch, dtype)
    (1000, 128, 7, torch.float16),      # partial last unit
    (63, 64, 1, torch.bfloat16),        # a single unit smaller than 64 rows
    (64 * 5, 64, 256, torch.float16),   # two M tiles, the full batch limit
    (4099, 256, 129, torch.bfloat16),   # two M tiles, one row in the second
    (148 * 64 * 9 + 17, 192, 33, torch.float16),  # every CTA walks three chunks
    (151936, 896, 64, torch.float16),   # Qwen2.5-0.5B: tied 151936 x 896 embedding, config 2's batch
]


@pytest.mark.parametrize("vocab,hidden,batch,dtype", SHAPES)
def test_matches_oracle(dev, ops, vocab, hidden, batch, dtype):
    h, w = _case(vocab, hidden, batch, dtype, dev, seed=vocab + batch)
    ws = ops.lm_head_argmax_workspace(batch, dev)
    top = torch.empty(batch, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = ops.lm_head_argmax(h, w, ws, max_logits=top, status=status)
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    amb = _check(ids, top, h, w, dtype)
    assert amb.sum() <= max(1, batch // 10)  # near-ties are rare: most rows are checked exactly
    assert int(ws.abs().sum()) == 0  # the workspace is left zeroed


def test_7b_lm_head_bf16(dev, ops):
    """Qwen2.5-7B's separate 152064 x 3584 bf16 lm_head."""
    h, w = _case(152064, 3584, 32, torch.bfloat16, dev, seed=7)
    ws = ops.lm_head_argmax_workspace(32, dev)
    top = torch.empty(32, dtype=torch.float32, device=dev)
    ids = ops.lm_head_argmax(h, w, ws, max_logits=top)
    _check(ids, top, h, w, torch.bfloat16)


@pytest.mark.parametrize("name", ["fp16_tied", "bf16"])
def test_golden_fixture(dev, ops, golden_dir, name):
    d = np.load(golden_dir / f"lm_head_{name}.npz")
    dtype = torch.float16 if str(d["dtype"]) == "float16" else torch.bfloat16
    h = torch.from_numpy(d["hidden"]).view(dtype).to(dev)
    w = torch.from_numpy(d["weight"]).view(dtype).to(dev)
    ws = ops.lm_head_argmax_workspace(h.shape[0], dev)
    top = torch.empty(h.shape[0], dtype=torch.float32, device=dev)
    ids = ops.lm_head_argmax(h, w, ws, max_logits=top)
    np.testing.assert_array_equal(ids.cpu().numpy(), d["tokens"])  # ties and the NaN row included
    ref = d["logits"]
    fin = np.isfinite(ref).all(axis=1)
    want = ref[fin].max(axis=1).astype(np.float64)
    assert (np.abs(top.cpu().numpy()[fin] - want) <= oracle.ulp(want, str(d["dtype"]))).all()
    assert np.isnan(top.cpu().numpy()[~fin]).all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_matches_torch_path_on_device(dev, ops, dtype):
    """The reference's compute_logits + argmax, run by torch (cuBLAS) on the same inputs."""
    h, w = _case(151936, 896, 48, dtype, dev, seed=3)
    ws = ops.lm_head_argmax_workspace(48, dev)
    ids = ops.lm_head_argmax(h, w, ws).cpu().numpy()
    ref = F.linear(h, w).float().argmax(dim=-1).cpu().numpy()
    exact = _exact(h, w)
    amb = oracle.ambiguous_rows(exact, NP_DTYPE[dtype])
    np.testing.assert_array_equal(ids[~amb], ref[~amb])
    assert oracle.acceptable(exact, NP_DTYPE[dtype], ids).all()


def test_exact_ties_pick_the_first_index(dev, ops):
    h, w = _case(5000, 256, 16, torch.float16, dev, seed=11)
    lead = (h[0].float() * 0.05).to(torch.float16)
    for v in (4999, 2500, 77, 4000):  # equal rows in different CTAs and chunks
        w[v] = lead
    ws = ops.lm_head_argmax_workspace(16, dev)
    ids = ops.lm_head_argmax(h, w, ws)
    assert int(ids[0]) == 77


def test_nan_row_returns_the_first_index(dev, ops):
    h, w = _case(3000, 128, 4, torch.bfloat16, dev, seed=12)
    h[2, 7] = float("nan")
    ws = ops.lm_head_argmax_workspace(4, dev)
    top = torch.empty(4, dtype=torch.float32, device=dev)
    ids = ops.lm_head_argmax(h, w, ws, max_logits=top)
    assert int(ids[2]) == 0 and torch.isnan(top[2])
    _check(ids[[0, 1, 3]], top[[0, 1, 3]], h[[0, 1, 3]], w, torch.bfloat16)


def test_workspace_reuse_and_strided_rows(dev, ops):
    """Back-to-back calls share a workspace; hidden may be a strided view (hidden[:, -1] of [B, T, H])."""
    _, w = _case(20000, 256, 1, torch.float16, dev, seed=13)
    ws = ops.lm_head_argmax_workspace(40, dev)
    g = torch.Generator(device="cpu").manual_seed(14)
    for batch in (40, 3, 17):
        seq = torch.randn(batch, 5, 256, generator=g).to(torch.float16).to(dev)
        h = seq[:, -1]
        assert h.stride(0) == 5 * 256
        ids = ops.lm_head_argmax(h, w, ws, weight_ready=True)
        _check(ids, None, h, w, torch.float16)
    assert int(ws.abs().sum()) == 0


def test_cuda_graph_replay(dev, ops):
    h, w = _case(151936, 896, 32, torch.float16, dev, seed=15)
    ws = ops.lm_head_argmax_workspace(32, dev)
    out = torch.empty(32, dtype=torch.int64, device=dev)
    ops.lm_head_argmax(h, w, ws, out=out, weight_ready=True)  # warm up (tensor maps, attributes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.lm_head_argmax(h, w, ws, out=out, weight_ready=True)
    g = torch.Generator(device="cpu").manual_seed(16)
    for _ in range(3):
        h.copy_(torch.randn(32, 896, generator=g).to(torch.float16))
        graph.replay()
        torch.cuda.synchronize()
        _check(out, None, h, w, torch.float16)


def test_greedy_lm_head_tokens(dev):
    from mini_inference_b200.sampler import GreedyLMHead
    h, w = _case(151936, 896, 8, torch.float16, dev, seed=17)
    head = GreedyLMHead(w, max_batch=64)
    toks = head.tokens(h)
    assert isinstance(toks, list) and len(toks) == 8
    _check(torch.tensor(toks), None, h, w, torch.float16)


def test_greedy_lm_head_slices_batches_above_the_kernel_limit(dev):
    """A batch of 300 rows (max_num_seqs above 256) goes through the kernel in slices of 256."""
    from mini_inference_b200.sampler import GreedyLMHead
    h, w = _case(4099, 256, 300, torch.float16, dev, seed=23)
    head = GreedyLMHead(w, max_batch=320)
    top = torch.empty(300, dtype=torch.float32, device=dev)
    ids = head(h, max_logits=top)
    torch.cuda.synchronize()
    _check(ids, top, h, w, torch.float16)
    assert int(head.workspace.abs().sum()) == 0


def test_rejects_unsupported_shapes(dev, ops):
    from mini_inference_b200 import PkvError
    ws = ops.lm_head_argmax_workspace(300, dev)
    h, w = _case(1000, 96, 4, torch.float16, dev, seed=18)  # hidden not a multiple of 64
    with pytest.raises(PkvError):
        ops.lm_head_argmax(h, w, ws)
    h, w = _case(1000, 128, 257, torch.float16, dev, seed=19)  # batch above 256
    with pytest.raises(PkvError):
        ops.lm_head_argmax(h, w, ws)
    h, w = _case(1000, 128, 8, torch.float16, dev, seed=20)
    with pytest.raises(PkvError):
        ops.lm_head_argmax(h, w, ws[:1])  # workspace too small
