"""Parity of the sm_100a kernels with the oracle and the reference's golden vectors (needs a B200).

Bars (north star): KV-cache writes, slot_mapping, block tables and positions
bit-exact; attention outputs within 2e-3 absolute of the oracle's exact result
in fp16, and within 2e-3 plus one bf16 step (2^-7 relative) in bf16, whose
values are spaced 2^-8 apart already in [0.5, 1).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.numerics import round_to, to_compute
from oracle.paged_kv import decode_attend, decode_metadata, packed_prefill_attend, write_index

pytestmark = pytest.mark.gpu

TOL = {"float16": (2e-3, 0.0), "bfloat16": (2e-3, 2.0 ** -7)}
# Against the reference's own CPU results the bf16 golden outputs are looser (its CPU SDPA
# rounds intermediates to bf16; see tests/test_oracle_golden.py).
GOLDEN_TOL = {"float16": (2e-3, 0.0), "bfloat16": (8e-3, 2.0 ** -7)}
TORCH = {"float16": torch.float16, "bfloat16": torch.bfloat16}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def excess(got: np.ndarray, ref: np.ndarray, dtype: str, tol=TOL) -> float:
    atol, rtol = tol[dtype]
    return float((np.abs(got - ref) - (atol + rtol * np.abs(ref))).max(initial=-1.0))


def to_torch(a: np.ndarray, dtype: str, dev) -> torch.Tensor:
    if dtype == "bfloat16":
        return torch.from_numpy(np.ascontiguousarray(a).astype(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def to_np(t: torch.Tensor) -> np.ndarray:
    """Exact values as float64 (bf16 via float32)."""
    return t.detach().float().cpu().numpy().astype(np.float64)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy()


def _tables_from(z) -> list[list[int]]:
    return [list(map(int, row[:n])) for row, n in zip(z["tables"], z["table_lens"])]


# ------------------------------------------------------------------ decode vs golden fixtures


@pytest.mark.parametrize("name", ["fp16_h14_d64", "bf16_h28_d128", "fp16_h28_d128"])
def test_decode_kernel_matches_golden(dev, golden_dir, name):
    from mini_inference_b200 import ops

    z = np.load(golden_dir / f"decode_{name}.npz")
    dt, layer, bs = str(z["dtype"]), int(z["layer"]), int(z["block_size"])
    k_pool = to_torch(z["k_before"], dt, dev)
    v_pool = to_torch(z["v_before"], dt, dev)
    tables = _tables_from(z)
    pos = z["positions"].astype(np.int64)
    meta = decode_metadata(tables, pos, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    q = to_torch(z["q"], dt, dev)
    k_new = to_torch(z["k_new"], dt, dev)
    v_new = to_torch(z["v_new"], dt, dev)
    pool = ops.make_pool(k_pool, v_pool)
    tabs = ops.make_tables(tab)
    ctx = torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev)
    slots = torch.from_numpy(meta["slot_mapping"]).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.decode_workspace_bytes(len(pos), k_pool.shape[2], tab.shape[1], bs, k_pool.shape[4],
                                                q.shape[1]), dtype=torch.uint8, device=dev)
    out = ops.decode_attention(pool, layer, tabs, q, ctx, ws, k_new=k_new, v_new=v_new, slot_mapping=slots,
                               status=status)
    ops.raise_device_errors(status)
    got = to_np(out)
    assert excess(got, to_compute(z["out"], dt).astype(np.float64), dt, GOLDEN_TOL) <= 0
    # Against the oracle (exact arithmetic, rounded to the storage type).
    kp = to_compute(z["k_before"], dt)[layer].copy()
    vp = to_compute(z["v_before"], dt)[layer].copy()
    ref = decode_attend(kp, vp, tables, pos.tolist(), to_compute(z["q"], dt), to_compute(z["k_new"], dt),
                        to_compute(z["v_new"], dt))
    assert excess(got, round_to(ref, dt), dt) <= 0
    # The append: the pool equals the reference's after-state bit for bit, in every layer.
    k_after = z["k_before"].copy()
    v_after = z["v_before"].copy()
    k_after[layer][z["k_written_at"][0], :, z["k_written_at"][1]] = z["k_written"]
    v_after[layer][z["v_written_at"][0], :, z["v_written_at"][1]] = z["v_written"]
    assert np.array_equal(bits(k_pool), k_after.view(np.int16))
    assert np.array_equal(bits(v_pool), v_after.view(np.int16))


@pytest.mark.parametrize("name", ["fp16_single", "fp16_packed", "fp16_prefix", "bf16_prefix_d128"])
def test_prefill_kernels_match_golden(dev, golden_dir, name):
    from mini_inference_b200 import ops

    z = np.load(golden_dir / f"prefill_{name}.npz")
    dt, bs = str(z["dtype"]), int(z["block_size"])
    k_pool = to_torch(z["k_before"], dt, dev)[None].contiguous()
    v_pool = to_torch(z["v_before"], dt, dev)[None].contiguous()
    tables = _tables_from(z)
    starts, lengths = z["starts"].astype(np.int64), z["lengths"].astype(np.int64)
    width = max(len(t) for t in tables)
    tab = np.full((len(tables), width), -1, np.int32)
    for i, t in enumerate(tables):
        tab[i, : len(t)] = t
    tab_d = torch.from_numpy(tab).to(dev)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)).to(dev)
    st = torch.from_numpy(starts.astype(np.int32)).to(dev)
    total = int(lengths.sum())
    pool = ops.make_pool(k_pool, v_pool)
    tabs = ops.make_tables(tab_d)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    positions = torch.empty(total, dtype=torch.int64, device=dev)
    slot_mapping = torch.empty(total, dtype=torch.int64, device=dev)
    ops.build_prefill_metadata(tabs, cu, st, bs, total, positions, slot_mapping, status)
    b, o = write_index(tables, starts.tolist(), lengths.tolist(), bs)
    assert positions.cpu().tolist() == z["positions"].tolist()
    assert slot_mapping.cpu().numpy().tolist() == (b * bs + o).tolist()
    q = to_torch(z["q"], dt, dev)  # [Hq, N, d]
    k = to_torch(z["k"], dt, dev)
    v = to_torch(z["v"], dt, dev)
    ops.kv_append(pool, 0, k.transpose(0, 1), v.transpose(0, 1), slot_mapping, status)
    out = ops.prefill_attention(pool, 0, tabs, q.transpose(0, 1), cu, st, int(lengths.max()), status=status)
    ops.raise_device_errors(status)
    got = to_np(out).transpose(1, 0, 2)  # -> [Hq, N, d]
    assert excess(got, to_compute(z["out"], dt).astype(np.float64), dt, GOLDEN_TOL) <= 0
    kp, vp = to_compute(z["k_before"], dt).copy(), to_compute(z["v_before"], dt).copy()
    ref = packed_prefill_attend(kp, vp, tables, starts.tolist(), lengths.tolist(), to_compute(z["q"], dt),
                                to_compute(z["k"], dt), to_compute(z["v"], dt))
    assert excess(got, round_to(ref, dt), dt) <= 0
    k_after = z["k_before"].copy()
    k_after[z["k_written_at"][0], :, z["k_written_at"][1]] = z["k_written"]
    v_after = z["v_before"].copy()
    v_after[z["v_written_at"][0], :, z["v_written_at"][1]] = z["v_written"]
    assert np.array_equal(bits(k_pool[0]), k_after.view(np.int16))
    assert np.array_equal(bits(v_pool[0]), v_after.view(np.int16))


@pytest.mark.parametrize("dtype,d", [("float16", 64), ("bfloat16", 128)])
def test_prefill_scores_growing_along_the_keys(dev, dtype, d):
    """Keys whose scores grow by far more than 2^8 from one 64-key stage to the next.

    The tensor-core prefill keeps a reference max per row and rescales its TMEM
    accumulator only when a row's max grows past it; random scores almost never do
    that, these force it at every stage, with a prefix hit and a query tile cut by
    the end of its sequence.
    """
    from mini_inference_b200 import ops

    rng = np.random.default_rng(11)
    hq, hkv, bs = 14, 2, 16
    starts, lengths = [200, 0], [77, 150]
    ends = [a + n for a, n in zip(starts, lengths)]
    nblk = [(e + bs - 1) // bs for e in ends]
    nb = sum(nblk) + 4
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in nblk:
        tables.append(perm[at:at + n].tolist())
        at += n
    kp = rng.standard_normal((nb + 1, hkv, bs, d)).astype(np.float32)
    vp = rng.standard_normal((nb + 1, hkv, bs, d)).astype(np.float32)
    q = rng.standard_normal((hq, sum(lengths), d)).astype(np.float32)
    # The score of the key at position p scales with 1 + p / 8: the row max grows along the keys.
    for table, e in zip(tables, ends):
        for pos in range(e):
            kp[table[pos // bs], :, pos % bs] *= 1.0 + pos / 8.0
    k_new = np.zeros((hkv, sum(lengths), d), np.float32)
    v_new = rng.standard_normal((hkv, sum(lengths), d)).astype(np.float32)
    t0 = 0
    for table, a, n in zip(tables, starts, lengths):
        for i in range(n):
            pos = a + i
            k_new[:, t0 + i] = rng.standard_normal((hkv, d)) * (1.0 + pos / 8.0)
        t0 += n
    tdt = TORCH[dtype]
    kq, vq, qq = round_to(kp, dtype), round_to(vp, dtype), round_to(q, dtype)
    knq, vnq = round_to(k_new, dtype), round_to(v_new, dtype)
    k_pool = torch.from_numpy(kq).to(tdt).to(dev)[None].contiguous()
    v_pool = torch.from_numpy(vq).to(tdt).to(dev)[None].contiguous()
    width = max(nblk)
    tab = np.full((len(tables), width), -1, np.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = t
    tabs = ops.make_tables(torch.from_numpy(tab).to(dev))
    pool = ops.make_pool(k_pool, v_pool)
    cu = torch.tensor([0, lengths[0], sum(lengths)], dtype=torch.int32, device=dev)
    st = torch.tensor(starts, dtype=torch.int32, device=dev)
    total = sum(lengths)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    positions = torch.empty(total, dtype=torch.int64, device=dev)
    slot_mapping = torch.empty(total, dtype=torch.int64, device=dev)
    ops.build_prefill_metadata(tabs, cu, st, bs, total, positions, slot_mapping, status)
    kt = torch.from_numpy(knq).to(tdt).to(dev)
    vt = torch.from_numpy(vnq).to(tdt).to(dev)
    ops.kv_append(pool, 0, kt.transpose(0, 1), vt.transpose(0, 1), slot_mapping, status)
    qt = torch.from_numpy(qq).to(tdt).to(dev)
    out = ops.prefill_attention(pool, 0, tabs, qt.transpose(0, 1), cu, st, max(lengths), status=status)
    ops.raise_device_errors(status)
    got = to_np(out).transpose(1, 0, 2)
    ref = packed_prefill_attend(kq.astype(np.float64), vq.astype(np.float64), tables, starts, lengths,
                                qq.astype(np.float64), knq.astype(np.float64), vnq.astype(np.float64))
    assert np.isfinite(got).all()
    assert excess(got, round_to(ref, dtype), dtype) <= 0


# ------------------------------------------------------------------ the micro-benchmark shape, full size


def micro_bench_case(dev, seed=0, batch=64, lo=128, hi=2048, num_blocks=16384, layers=2, dtype=torch.float16,
                     hq=14, hkv=2, d=64):
    """The task's configuration 2: 64 sequences, context U{128..2048}, tables from a seeded permutation of the pool."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(lo, hi + 1, (batch,), generator=g)
    perm = torch.randperm(num_blocks, generator=g)
    bs = 16
    tables, at = [], 0
    for c in ctx.tolist():
        nb = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + nb].tolist())
        at += nb
    shape = (layers, num_blocks + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    v_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    q = torch.randn(batch, hq, d, generator=g).to(dtype).to(dev)
    k_new = torch.randn(batch, hkv, d, generator=g).to(dtype).to(dev)
    v_new = torch.randn(batch, hkv, d, generator=g).to(dtype).to(dev)
    return ctx.tolist(), tables, k_pool, v_pool, q, k_new, v_new


@pytest.mark.parametrize("dtype,hq,hkv,d", [(torch.float16, 14, 2, 64), (torch.bfloat16, 28, 4, 128)])
def test_decode_full_size_matches_oracle(dev, dtype, hq, hkv, d):
    from mini_inference_b200 import ops

    batch = 64 if d == 64 else 16
    ctx, tables, k_pool, v_pool, q, k_new, v_new = micro_bench_case(dev, seed=1, batch=batch, dtype=dtype, hq=hq,
                                                                    hkv=hkv, d=d, num_blocks=8192 if d == 128 else 16384)
    bs = 16
    layer = 1
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    k_before = k_pool[layer].clone()
    pool = ops.make_pool(k_pool, v_pool)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.decode_workspace_bytes(batch, hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8, device=dev)
    ctx_lens = torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev)
    slots = torch.from_numpy(meta["slot_mapping"]).to(dev)
    out = ops.decode_attention(pool, layer, ops.make_tables(tab), q, ctx_lens, ws, k_new=k_new, v_new=v_new,
                               slot_mapping=slots, status=status)
    # A second call on the same workspace gives the same bits (the split-K tickets were reset).
    out2 = ops.decode_attention(pool, layer, ops.make_tables(tab), q, ctx_lens, ws, k_new=k_new, v_new=v_new,
                                slot_mapping=slots, status=status)
    ops.raise_device_errors(status)
    assert torch.equal(out, out2)
    name = "float16" if dtype == torch.float16 else "bfloat16"
    kp = to_np(k_before)
    vp = to_np(v_pool[layer]).copy()  # after the append; the oracle's append rewrites the same rows
    ref = decode_attend(kp.copy(), vp, tables, ctx, to_np(q), to_np(k_new), to_np(v_new))
    assert excess(to_np(out), round_to(ref, name), name) <= 0
    # Append bit-exact: only the rows at slot_mapping changed, to k_new.
    k_after = k_pool[layer].cpu()
    exp = k_before.cpu().clone()
    sm = meta["slot_mapping"]
    exp[torch.from_numpy(sm // bs), :, torch.from_numpy(sm % bs)] = k_new.cpu()
    assert torch.equal(k_after.view(torch.int16), exp.view(torch.int16))


def test_decode_edge_lengths(dev):
    """Block boundaries, one-key sequences, one chunk vs many, and the longest table."""
    from mini_inference_b200 import ops

    bs, hq, hkv, d = 16, 14, 2, 64
    ctx = [0, 1, 14, 15, 16, 17, 31, 32, 127, 128, 129, 255, 256, 257, 1023, 2047]
    g = torch.Generator().manual_seed(5)
    nb = sum((c + 1 + bs - 1) // bs for c in ctx) + 3
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).half().to(dev)
    v_pool = torch.randn(shape, generator=g).half().to(dev)
    q = torch.randn(len(ctx), hq, d, generator=g).half().to(dev)
    kn = torch.randn(len(ctx), hkv, d, generator=g).half().to(dev)
    vn = torch.randn(len(ctx), hkv, d, generator=g).half().to(dev)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables) + 3, pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    pool = ops.make_pool(k_pool, v_pool)
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    out = ops.decode_attention(pool, 0, ops.make_tables(tab),
                               q, torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws, k_new=kn,
                               v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    ops.raise_device_errors(status)
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, "float16"), "float16") <= 0


def test_decode_without_append_and_with_strided_inputs(dev):
    """q/k/v as the model hands them over: transposed views of one fused qkv row."""
    from mini_inference_b200 import ops

    bs, hq, hkv, d = 16, 14, 2, 64
    ctx, tables, k_pool, v_pool, _, _, _ = micro_bench_case(dev, seed=3, batch=8, lo=1, hi=300, num_blocks=256,
                                                            layers=1)
    qkv = torch.randn(8, 1, (hq + 2 * hkv) * d, device=dev).half()
    q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    q = q.view(8, 1, hq, d).transpose(1, 2)  # [B, Hq, 1, d], non-contiguous
    k = k.view(8, 1, hkv, d).transpose(1, 2)
    v = v.view(8, 1, hkv, d).transpose(1, 2)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    pool = ops.make_pool(k_pool, v_pool)
    ws = torch.zeros(ops.decode_workspace_bytes(8, hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8, device=dev)
    ctx_lens = torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev)
    slots = torch.from_numpy(meta["slot_mapping"]).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    ops.kv_append(pool, 0, k[:, :, 0], v[:, :, 0], slots, status)  # standalone append, strided rows
    out = ops.decode_attention(pool, 0, ops.make_tables(tab), q[:, :, 0], ctx_lens, ws, status=status)
    ops.raise_device_errors(status)
    ref = decode_attend(kp, vp, tables, ctx, to_np(q[:, :, 0]), to_np(k[:, :, 0]), to_np(v[:, :, 0]))
    assert excess(to_np(out), round_to(ref, "float16"), "float16") <= 0


def test_out_of_range_block_is_reported_not_faulted(dev):
    """A block id past the pool is recorded in the status word; the load is clamped, no fault."""
    from mini_inference_b200 import ops

    k_pool = torch.zeros(1, 5, 2, 16, 64, dtype=torch.float16, device=dev)
    v_pool = torch.zeros_like(k_pool)
    tab = torch.tensor([[1, 99]], dtype=torch.int32, device=dev)
    q = torch.randn(1, 14, 64, device=dev).half()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(ops.decode_workspace_bytes(1, 2, 2, 16, 64, 14), dtype=torch.uint8, device=dev)
    ops.decode_attention(ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q,
                         torch.tensor([20], dtype=torch.int32, device=dev), ws, status=status)
    with pytest.raises(IndexError):
        ops.raise_device_errors(status)
    torch.cuda.synchronize()  # the context is still usable


# ------------------------------------------------------------------ metadata builder and block copy


def test_decode_metadata_builder_matches_oracle(dev):
    from mini_inference_b200 import ops

    rng = np.random.default_rng(0)
    rows, cols, bs = 10, 12, 16
    mirror = rng.integers(0, 500, (rows, cols)).astype(np.int32)
    seq_rows = np.array([3, 0, -1, 9, 5, -1], np.int32)
    lengths = np.array([0, 15, 0, 16, 191, 0], np.int32)
    tabs_d = torch.from_numpy(mirror).to(dev)
    sr = torch.from_numpy(seq_rows).to(dev)
    ln = torch.from_numpy(lengths).to(dev)
    pos = torch.empty(6, dtype=torch.int64, device=dev)
    sm = torch.empty(6, dtype=torch.int64, device=dev)
    cl = torch.empty(6, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.build_decode_metadata(ops.make_tables(tabs_d, sr), ln, bs, 777, pos, sm, cl, status)
    ops.raise_device_errors(status)
    real = seq_rows >= 0
    tables = [mirror[r].tolist() for r in seq_rows[real]]
    meta = decode_metadata(tables, lengths[real], bs, cols, pad_block=777)
    assert pos.cpu().numpy()[real].tolist() == meta["positions"].tolist()
    assert sm.cpu().numpy()[real].tolist() == meta["slot_mapping"].tolist()
    assert cl.cpu().numpy()[real].tolist() == meta["context_lens"].tolist()
    # CUDA-graph padding rows: position 0 of the scratch block, one key.
    assert sm.cpu().numpy()[~real].tolist() == [777 * bs] * 2 and cl.cpu().numpy()[~real].tolist() == [1, 1]


def test_table_mirror_updates_and_commit(dev):
    from mini_inference_b200 import ops

    tabs = torch.full((4, 5), -1, dtype=torch.int32, device=dev)
    upd = torch.tensor([[0, 0, 7], [0, 1, 9], [3, 4, 2], [2, 0, 11]], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.update_tables(tabs, upd, status)
    ops.raise_device_errors(status)
    exp = torch.full((4, 5), -1, dtype=torch.int32)
    exp[0, 0], exp[0, 1], exp[3, 4], exp[2, 0] = 7, 9, 2, 11
    assert torch.equal(tabs.cpu(), exp)
    lengths = torch.tensor([5, 0, 3, 8], dtype=torch.int32, device=dev)
    ops.commit_decode(torch.tensor([3, -1, 0], dtype=torch.int32, device=dev), lengths)
    assert lengths.cpu().tolist() == [6, 0, 3, 9]


def test_copy_blocks_is_exact(dev):
    from mini_inference_b200 import ops

    k = torch.randn(3, 9, 2, 16, 64, device=dev).half()
    v = torch.randn_like(k)
    k0, v0 = k.clone(), v.clone()
    src = torch.tensor([1, 4, 8], dtype=torch.int32, device=dev)
    dst = torch.tensor([2, 0, 5], dtype=torch.int32, device=dev)
    ops.copy_blocks(ops.make_pool(k, v), src, dst)
    ek, ev = k0.clone(), v0.clone()
    for s_, d_ in zip(src.tolist(), dst.tolist()):
        ek[:, d_] = k0[:, s_]
        ev[:, d_] = v0[:, s_]
    assert torch.equal(k, ek) and torch.equal(v, ev)


def test_decode_graph_replays_stay_exact(dev):
    """Hundreds of back-to-back replays of a multi-layer decode graph: no device error, and
    every replay returns the bits of the first eager call (split-K merge order is fixed).
    Layers after the first start their block lookups before the previous kernel ends
    (PKV_DECODE_INPUTS_READY), which must not change a bit.

    Regression test for ring-stage phase tracking: a consumer that skips a stage's use can
    mistake a phase two ahead for the one it waits on, which only shows under replay timing.
    """
    from mini_inference_b200 import ops

    layers, bs, hq, hkv, d = 4, 16, 14, 2, 64
    ctx, tables, k_pool, v_pool, q, k_new, v_new = micro_bench_case(dev, seed=7, layers=layers)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    pool = ops.make_pool(k_pool, v_pool)
    tabs = ops.make_tables(tab)
    ctx_lens = torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev)
    slots = torch.from_numpy(meta["slot_mapping"]).to(dev)
    ws = torch.zeros(ops.decode_workspace_bytes(64, hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = torch.empty(layers, 64, hq, d, dtype=torch.float16, device=dev)

    def step():
        for layer in range(layers):
            ops.decode_attention(pool, layer, tabs, q, ctx_lens, ws, k_new=k_new, v_new=v_new, slot_mapping=slots,
                                 out=outs[layer], status=status, inputs_ready=layer > 0)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    first = outs.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(300):
        graph.replay()
    torch.cuda.synchronize()
    ops.raise_device_errors(status)
    assert torch.equal(outs, first)


@pytest.mark.parametrize("dtype,hq,hkv,d,ctx", [(torch.float16, 14, 2, 64, [4000]), (torch.bfloat16, 28, 4, 128, [3000, 37]),
                                              # the 7B long-context shape (config 5): tens of chunks per sequence
                                              (torch.bfloat16, 28, 4, 128, [16000, 5000, 24000])])
def test_decode_few_long_sequences_split_over_many_ctas(dev, dtype, hq, hkv, d, ctx):
    """A batch of one or two long sequences is spread over every CTA, so each is merged from
    more pieces than the merging CTA can stage at once (the multi-round merge path)."""
    from mini_inference_b200 import ops

    bs = 16
    g = torch.Generator().manual_seed(11)
    nb = sum((c + 1 + bs - 1) // bs for c in ctx) + 1
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    v_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    q = torch.randn(len(ctx), hq, d, generator=g).to(dtype).to(dev)
    kn = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    vn = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    out = ops.decode_attention(ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q,
                               torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws, k_new=kn,
                               v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    ops.raise_device_errors(status)
    name = "float16" if dtype == torch.float16 else "bfloat16"
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, name), name) <= 0


def test_chunked_prefill_matches_one_shot(dev):
    """A long prompt prefilled in chunks (each chunk attends to the cached earlier ones) = one pass.

    The varlen kernel takes any start per sequence, so chunked prefill (listed as missing in
    the reference, README.md:470-473) is a scheduling choice: the pools come out bit-identical
    and the outputs agree within the attention tolerance.
    """
    from mini_inference_b200 import PagedKVCache

    hq, hkv, d = 14, 2, 64
    n, chunks = 300, [128, 100, 72]
    g = torch.Generator(device=dev).manual_seed(21)
    q = torch.randn(1, hq, n, d, generator=g, device=dev).half()
    k = torch.randn(1, hkv, n, d, generator=g, device=dev).half()
    v = torch.randn(1, hkv, n, d, generator=g, device=dev).half()
    caches = [PagedKVCache(1, hkv, d, num_blocks=32, block_size=16, max_seqs=2, max_len=512, dtype=torch.float16,
                           device=dev) for _ in range(2)]
    one, chunked = caches
    s1 = one.allocate(n)
    ctx = one.packed_prefill_context([s1], [n])
    out_one = ctx.attend(0, q, k, v)
    ctx.commit()
    s2 = chunked.allocate(chunks[0])
    outs, at = [], 0
    for c in chunks:
        ctx = chunked.packed_prefill_context([s2], [c])
        outs.append(ctx.attend(0, q[:, :, at:at + c], k[:, :, at:at + c], v[:, :, at:at + c]))
        ctx.commit()
        at += c
    one.raise_device_errors(), chunked.raise_device_errors()
    assert chunked.lengths[s2] == one.lengths[s1] == n
    assert chunked.block_tables[s2] == one.block_tables[s1]
    assert torch.equal(chunked.k, one.k) and torch.equal(chunked.v, one.v)
    torch.testing.assert_close(torch.cat(outs, dim=2), out_one, atol=2e-3, rtol=2e-3)


def test_prefill_more_sequences_than_one_launch_holds(dev):
    """2100 short sequences (some without new tokens): the host splits them over two persistent launches."""
    from mini_inference_b200 import ops

    rng = np.random.default_rng(13)
    hq, hkv, d, bs = 14, 2, 64, 16
    n_seq = 2100
    lengths = rng.integers(0, 4, n_seq).tolist()  # 0..3 new tokens
    starts = rng.integers(0, 20, n_seq).tolist()
    ends = [a + n for a, n in zip(starts, lengths)]
    nblk = [max(1, (e + bs - 1) // bs) for e in ends]
    nb = sum(nblk) + 2
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in nblk:
        tables.append(perm[at:at + n].tolist())
        at += n
    kp = rng.standard_normal((nb + 1, hkv, bs, d)).astype(np.float32)
    vp = rng.standard_normal((nb + 1, hkv, bs, d)).astype(np.float32)
    total = sum(lengths)
    q = rng.standard_normal((hq, total, d)).astype(np.float32)
    k_new = rng.standard_normal((hkv, total, d)).astype(np.float32)
    v_new = rng.standard_normal((hkv, total, d)).astype(np.float32)
    kq, vq, qq = round_to(kp, "float16"), round_to(vp, "float16"), round_to(q, "float16")
    knq, vnq = round_to(k_new, "float16"), round_to(v_new, "float16")
    k_pool = torch.from_numpy(kq).half().to(dev)[None].contiguous()
    v_pool = torch.from_numpy(vq).half().to(dev)[None].contiguous()
    tab = np.full((n_seq, max(nblk)), -1, np.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = t
    tabs = ops.make_tables(torch.from_numpy(tab).to(dev))  # no seq_rows: row = sequence index
    pool = ops.make_pool(k_pool, v_pool)
    cu = torch.tensor([0] + np.cumsum(lengths).tolist(), dtype=torch.int32, device=dev)
    st = torch.tensor(starts, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    positions = torch.empty(total, dtype=torch.int64, device=dev)
    slot_mapping = torch.empty(total, dtype=torch.int64, device=dev)
    ops.build_prefill_metadata(tabs, cu, st, bs, total, positions, slot_mapping, status)
    ops.kv_append(pool, 0, torch.from_numpy(knq).half().to(dev).transpose(0, 1),
                  torch.from_numpy(vnq).half().to(dev).transpose(0, 1), slot_mapping, status)
    qt = torch.from_numpy(qq).half().to(dev)
    out = ops.prefill_attention(pool, 0, tabs, qt.transpose(0, 1), cu, st, max(lengths), status=status)
    ops.raise_device_errors(status)
    got = to_np(out).transpose(1, 0, 2)
    ref = packed_prefill_attend(kq.astype(np.float64), vq.astype(np.float64), tables, starts, lengths,
                                qq.astype(np.float64), knq.astype(np.float64), vnq.astype(np.float64))
    assert np.isfinite(got).all()
    assert excess(got, round_to(ref, "float16"), "float16") <= 0


def test_decode_many_short_sequences_beside_long_ones_twice(dev):
    """1000 sequences: most of one block, ten long ones spread through the batch, so CTA ranges
    cover dozens of whole sequences next to cut ones. Two calls on one workspace give the
    same bits (every cut sequence's tickets came back to zero) and match the oracle."""
    from mini_inference_b200 import ops

    bs, hq, hkv, d = 16, 14, 2, 64
    g = torch.Generator().manual_seed(17)
    batch = 1000
    ctx = torch.randint(1, 16, (batch,), generator=g).tolist()
    for i in range(10):
        ctx[37 + 96 * i] = int(torch.randint(1500, 2001, (1,), generator=g))
    nb = sum((c + 1 + bs - 1) // bs for c in ctx) + 3
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).half().to(dev)
    v_pool = torch.randn(shape, generator=g).half().to(dev)
    q = torch.randn(batch, hq, d, generator=g).half().to(dev)
    kn = torch.randn(batch, hkv, d, generator=g).half().to(dev)
    vn = torch.randn(batch, hkv, d, generator=g).half().to(dev)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    pool = ops.make_pool(k_pool, v_pool)
    ws = torch.zeros(ops.decode_workspace_bytes(batch, hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    args = (pool, 0, ops.make_tables(tab), q, torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws)
    kw = dict(k_new=kn, v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    out = ops.decode_attention(*args, **kw)
    out2 = ops.decode_attention(*args, **kw)
    ops.raise_device_errors(status)
    assert torch.equal(out, out2)
    assert int(ws[:4096].view(torch.int32).abs().sum()) == 0
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, "float16"), "float16") <= 0


# Equal-range layouts at the 7B shape. "ragged": eight 36-41 K-token sequences. "on_bounds":
# 19240 blocks = 148 ranges of 130, sequences 1 and 2 starting exactly on range starts
# (blocks 1300 and 3900) and last blocks partly filled.
_ON_BOUNDS = [1300, 2600, 2500, 2400, 2600, 2500, 2700, 2640]
EQUAL_RANGE_LAYOUTS = {
    "ragged": [40000, 38000, 39000, 41000, 37000, 40000, 36000, 39500],
    "on_bounds": [16 * n - 1 - (3 * i) % 16 for i, n in enumerate(_ON_BOUNDS)],
}


@pytest.mark.parametrize("layout", sorted(EQUAL_RANGE_LAYOUTS))
def test_decode_equal_ranges_at_the_7b_shape(dev, layout):
    """Enough blocks (at least 128 per CTA) for the equal-range split at the 7B shape (bf16,
    Hq 28 / Hkv 4 / d 128): every CTA a range that cuts sequences anywhere, sequences that
    start on a range's first block among them (block 0 always does); twice on one workspace
    (the counters come back to zero), against the oracle."""
    from mini_inference_b200 import ops

    bs, hq, hkv, d = 16, 28, 4, 128
    ctx = EQUAL_RANGE_LAYOUTS[layout]
    g = torch.Generator().manual_seed(29)
    nb = sum((c + 1 + bs - 1) // bs for c in ctx) + 1
    assert nb >= 128 * torch.cuda.get_device_properties(dev).multi_processor_count  # the rule's threshold
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).bfloat16().to(dev)
    v_pool = torch.randn(shape, generator=g).bfloat16().to(dev)
    q = torch.randn(len(ctx), hq, d, generator=g).bfloat16().to(dev)
    kn = torch.randn(len(ctx), hkv, d, generator=g).bfloat16().to(dev)
    vn = torch.randn(len(ctx), hkv, d, generator=g).bfloat16().to(dev)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    args = (ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q,
            torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws)
    kw = dict(k_new=kn, v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    out = ops.decode_attention(*args, **kw)
    out2 = ops.decode_attention(*args, **kw)
    ops.raise_device_errors(status)
    assert torch.equal(out, out2)
    assert int(ws[:4096].view(torch.int32).abs().sum()) == 0
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, "bfloat16"), "bfloat16") <= 0


# Head layouts beyond the configs' 7-query groups: one KV head (8 warps per head, three
# pairwise merge rounds), eight (one warp per head, no merge), groups of 16 (16 MMA rows)
# and of 1.
HEAD_LAYOUTS = [(torch.float16, 16, 1, 64), (torch.bfloat16, 8, 1, 128), (torch.bfloat16, 64, 8, 128),
                (torch.float16, 8, 8, 64), (torch.float16, 32, 2, 128), (torch.bfloat16, 64, 4, 64)]


@pytest.mark.parametrize("dtype,hq,hkv,d", HEAD_LAYOUTS)
def test_decode_head_layouts(dev, dtype, hq, hkv, d):
    """Every KV-head count and group size the kernel takes, on short and cut sequences (the
    warps of a head merge, then the CTAs of a sequence), twice on one workspace, against the
    oracle."""
    from mini_inference_b200 import ops

    bs = 16
    ctx = [1, 15, 16, 17, 40, 100, 333, 700, 1500, 3000]
    g = torch.Generator().manual_seed(hq * 31 + hkv * 7 + d)
    nb = sum((c + 1 + bs - 1) // bs for c in ctx) + 2
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        n = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    v_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    q = torch.randn(len(ctx), hq, d, generator=g).to(dtype).to(dev)
    kn = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    vn = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    meta = decode_metadata(tables, ctx, bs, max(len(t) for t in tables), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    args = (ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q,
            torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws)
    kw = dict(k_new=kn, v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    out = ops.decode_attention(*args, **kw)
    out2 = ops.decode_attention(*args, **kw)
    ops.raise_device_errors(status)
    assert torch.equal(out, out2)
    assert int(ws[:4096].view(torch.int32).abs().sum()) == 0
    name = "float16" if dtype == torch.float16 else "bfloat16"
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, name), name) <= 0


def test_decode_serving_batch_takes_a_candidate_cap(dev):
    """190 sequences of log-uniform 56..1064 tokens (config 3's decode batch early on): more
    sequences than half the CTAs, where the split takes the smallest listed chunk cap whose
    units fill at most 29/32 of the CTAs. The same rule restated here must pick one (so the
    test covers that path); two calls on one workspace give the same bits and match the oracle."""
    from mini_inference_b200 import ops

    bs, hq, hkv, d, batch = 16, 14, 2, 64, 190
    g = torch.Generator().manual_seed(23)
    ctx = torch.exp(torch.empty(batch).uniform_(np.log(56.0), np.log(1064.0), generator=g)).long().tolist()
    nblk = [(c + 1 + bs - 1) // bs for c in ctx]
    ctas = 2 * torch.cuda.get_device_properties(dev).multi_processor_count
    caps = [12, 13, 14, 15, 16, 18, 20, 22, 24, 26, 28, 32, 36, 40, 48, 64]
    fit = [c for c in caps if sum(-(-n // c) for n in nblk) <= ctas * 29 // 32]
    assert batch > ctas // 2 and fit and any(n > fit[0] for n in nblk)  # a candidate is taken and cuts
    nb = sum(nblk) + 1
    perm = torch.randperm(nb, generator=g).tolist()
    tables, at = [], 0
    for n in nblk:
        tables.append(perm[at: at + n])
        at += n
    shape = (1, nb + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).half().to(dev)
    v_pool = torch.randn(shape, generator=g).half().to(dev)
    q = torch.randn(batch, hq, d, generator=g).half().to(dev)
    kn = torch.randn(batch, hkv, d, generator=g).half().to(dev)
    vn = torch.randn(batch, hkv, d, generator=g).half().to(dev)
    meta = decode_metadata(tables, ctx, bs, max(nblk), pad_block=0)
    tab = torch.from_numpy(meta["block_tables"].astype(np.int32)).to(dev)
    ws = torch.zeros(ops.decode_workspace_bytes(batch, hkv, tab.shape[1], bs, d, hq), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kp, vp = to_np(k_pool[0]), to_np(v_pool[0])
    args = (ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q,
            torch.from_numpy(meta["context_lens"].astype(np.int32)).to(dev), ws)
    kw = dict(k_new=kn, v_new=vn, slot_mapping=torch.from_numpy(meta["slot_mapping"]).to(dev), status=status)
    out = ops.decode_attention(*args, **kw)
    out2 = ops.decode_attention(*args, **kw)
    ops.raise_device_errors(status)
    assert torch.equal(out, out2)
    assert int(ws[:4096].view(torch.int32).abs().sum()) == 0
    ref = decode_attend(kp, vp, tables, ctx, to_np(q), to_np(kn), to_np(vn))
    assert excess(to_np(out), round_to(ref, "float16"), "float16") <= 0
