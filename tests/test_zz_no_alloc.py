"""pkv_decode_attention_static, the decode entry point that allocates nothing (needs a B200).

It runs the same kernel as pkv_decode_attention with the library's static
per-device scratch in place of a caller workspace, so two calls in a row must
give the same bits as two calls of the workspace entry point on the same
inputs: outputs and pool writes alike. The second pair also shows that the
scratch's ticket counters came back to zero. This file is collected last and
needs nothing from the other test files, so it passes alone and after them.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def _case(dev, seed, batch, hq, hkv, d, dtype, num_blocks):
    """Context lengths U{128..2048} (long ones split over many CTAs), tables from a seeded permutation."""
    g = torch.Generator().manual_seed(seed)
    bs = 16
    ctx = torch.randint(128, 2049, (batch,), generator=g).tolist()
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, at = [], 0
    for c in ctx:
        nb = (c + 1 + bs - 1) // bs
        tables.append(perm[at: at + nb])
        at += nb
    cols = max(len(t) for t in tables)
    tab = torch.zeros(batch, cols, dtype=torch.int32)
    for i, t in enumerate(tables):
        tab[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    slots = torch.tensor([t[c // bs] * bs + c % bs for t, c in zip(tables, ctx)], dtype=torch.int64)
    shape = (2, num_blocks + 1, hkv, bs, d)
    k_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    v_pool = torch.randn(shape, generator=g).to(dtype).to(dev)
    qs = [torch.randn(batch, hq, d, generator=g).to(dtype).to(dev) for _ in range(2)]
    news = [(torch.randn(batch, hkv, d, generator=g).to(dtype).to(dev),
             torch.randn(batch, hkv, d, generator=g).to(dtype).to(dev)) for _ in range(2)]
    ctx_lens = torch.tensor([c + 1 for c in ctx], dtype=torch.int32, device=dev)
    return tab.to(dev), slots.to(dev), ctx_lens, k_pool, v_pool, qs, news


@pytest.mark.parametrize("dtype,hq,hkv,d,batch,num_blocks",
                         [(torch.float16, 14, 2, 64, 64, 16384), (torch.bfloat16, 28, 4, 128, 16, 4096)])
def test_static_entry_point_matches_workspace_entry_point(dev, dtype, hq, hkv, d, batch, num_blocks):
    from mini_inference_b200 import ops

    tab, slots, ctx_lens, k_pool, v_pool, qs, news = _case(dev, 7, batch, hq, hkv, d, dtype, num_blocks)
    k_ws, v_ws = k_pool.clone(), v_pool.clone()  # the workspace entry point's own copy of the pool
    pool_static, pool_ws = ops.make_pool(k_pool, v_pool), ops.make_pool(k_ws, v_ws)
    tables = ops.make_tables(tab)
    ws = torch.zeros(ops.decode_workspace_bytes(batch, hkv, tab.shape[1], 16, d, hq), dtype=torch.uint8,
                     device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    outs = [torch.empty(batch, hq, d, dtype=dtype, device=dev) for _ in range(2)]
    layer = 1
    for call in range(2):
        q, (k_new, v_new) = qs[call], news[call]
        if call == 1:  # after the first call's set-up the static path claims no device memory
            torch.cuda.synchronize()
            allocated, free = torch.cuda.memory_allocated(dev), torch.cuda.mem_get_info(dev)[0]
        got = ops.decode_attention_static(pool_static, layer, tables, q, ctx_lens, outs[call], k_new=k_new,
                                          v_new=v_new, slot_mapping=slots, status=status[0:1])
        if call == 1:
            torch.cuda.synchronize()
            assert torch.cuda.memory_allocated(dev) == allocated
            assert torch.cuda.mem_get_info(dev)[0] == free
        want = ops.decode_attention(pool_ws, layer, tables, q, ctx_lens, ws, k_new=k_new, v_new=v_new,
                                    slot_mapping=slots, status=status[1:2])
        ops.raise_device_errors(status[0:1])
        ops.raise_device_errors(status[1:2])
        assert got.data_ptr() == outs[call].data_ptr()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"call {call}"
        assert torch.equal(k_pool.view(torch.int16), k_ws.view(torch.int16)), f"call {call}"
        assert torch.equal(v_pool.view(torch.int16), v_ws.view(torch.int16)), f"call {call}"


def test_static_entry_point_refuses_copies(dev):
    """The wrapper copies nothing: a strided last dimension is an error, not a hidden copy."""
    from mini_inference_b200 import ops

    tab, slots, ctx_lens, k_pool, v_pool, qs, _ = _case(dev, 3, 4, 14, 2, 64, torch.float16, 1024)
    out = torch.empty(4, 14, 64, dtype=torch.float16, device=dev)
    q_strided = torch.empty(4, 14, 128, dtype=torch.float16, device=dev)[:, :, ::2]
    with pytest.raises(ValueError, match="copies nothing"):
        ops.decode_attention_static(ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), q_strided, ctx_lens,
                                    out)


class _DeviceArray:
    """A raw device address as a torch tensor, through the CUDA array interface (no copy)."""

    def __init__(self, address: int, n: int, typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (address, False), "version": 2}


def test_static_reset_clears_stale_tickets(dev):
    """Tickets left in the static scratch (written here from the host) are cleared by the reset,
    after which the static entry point again matches the workspace entry point bit for bit."""
    from mini_inference_b200 import ops

    tab, slots, ctx_lens, k_pool, v_pool, qs, news = _case(dev, 11, 64, 14, 2, 64, torch.float16, 16384)
    out = torch.empty(64, 14, 64, dtype=torch.float16, device=dev)
    pool = ops.make_pool(k_pool, v_pool)
    tables = ops.make_tables(tab)
    ops.decode_attention_static(pool, 0, tables, qs[0], ctx_lens, out)  # set-up on this device
    torch.cuda.synchronize()
    addr, nbytes = ops.decode_static_scratch()
    assert addr and nbytes == 16 * 1024 * 1024
    tickets = torch.as_tensor(_DeviceArray(addr, 1024, "<i4"), device=dev)
    tickets[:64] = 3  # a stale ticket for every sequence of the batch
    ops.decode_static_reset()
    torch.cuda.synchronize()
    assert int(tickets.abs().sum()) == 0
    ws = torch.zeros(ops.decode_workspace_bytes(64, 2, tab.shape[1], 16, 64, 14), dtype=torch.uint8, device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    got = ops.decode_attention_static(pool, 0, tables, qs[1], ctx_lens, out, status=status[0:1])
    want = ops.decode_attention(pool, 0, tables, qs[1], ctx_lens, ws, status=status[1:2])
    ops.raise_device_errors(status[0:1])
    ops.raise_device_errors(status[1:2])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_static_entry_point_refuses_a_shape_beyond_the_scratch(dev):
    """8 KV heads of 16 query heads at head_dim 128 need ~20 MB of scratch on a 148-SM B200: the
    call is refused with PKV_ERR_WORKSPACE before anything runs, leaving out and status as they were."""
    from mini_inference_b200 import ops
    from mini_inference_b200._lib import PKV_ERR_WORKSPACE, PkvError

    if torch.cuda.get_device_properties(dev).multi_processor_count < 148:
        pytest.skip("the scratch need depends on the SM count; sized here for a 148-SM B200")
    tab, slots, ctx_lens, k_pool, v_pool, qs, _ = _case(dev, 5, 2, 128, 8, 128, torch.bfloat16, 512)
    out = torch.full((2, 128, 128), 7.0, dtype=torch.bfloat16, device=dev)
    status = torch.full((1,), 0, dtype=torch.int32, device=dev)
    before = out.clone()
    with pytest.raises(PkvError) as err:
        ops.decode_attention_static(ops.make_pool(k_pool, v_pool), 0, ops.make_tables(tab), qs[0], ctx_lens, out,
                                    status=status)
    assert err.value.status == PKV_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert torch.equal(out, before) and int(status.item()) == 0
