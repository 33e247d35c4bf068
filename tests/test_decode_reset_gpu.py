"""A decode workspace with stale ticket counters is made clean again (needs a B200).

Every decode call leaves its workspace's ticket counters at zero. A call that reported an
error may not have; the cache then zeroes them before the error propagates, and callers of
the C ABI use ``pkv_decode_reset_workspace``. The stale state is written here from the host
(no kernel is made to fail), then the reset runs and the next call must equal a call on a
fresh workspace bit for bit.
"""

from __future__ import annotations

import pytest
import torch

from tests.test_zz_no_alloc import _case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def test_reset_workspace_then_decode_matches_a_fresh_workspace(dev):
    from mini_inference_b200 import ops

    tab, slots, ctx_lens, k_pool, v_pool, qs, news = _case(dev, 21, 64, 14, 2, 64, torch.float16, 16384)
    pool, tables = ops.make_pool(k_pool, v_pool), ops.make_tables(tab)
    nbytes = ops.decode_workspace_bytes(64, 2, tab.shape[1], 16, 64, 14)
    fresh = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    stale = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    stale[:4096].view(torch.int32)[:64] = 2  # a stale ticket for every sequence
    ops.decode_reset_workspace(stale)
    torch.cuda.synchronize()
    assert int(stale[:4096].view(torch.int32).abs().sum()) == 0
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    got = ops.decode_attention(pool, 1, tables, qs[0], ctx_lens, stale, status=status[0:1])
    want = ops.decode_attention(pool, 1, tables, qs[0], ctx_lens, fresh, status=status[1:2])
    ops.raise_device_errors(status[0:1])
    ops.raise_device_errors(status[1:2])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_cache_clears_its_workspaces_when_it_raises(dev):
    from mini_inference_b200 import PagedKVCache

    cache = PagedKVCache(2, 2, 64, num_blocks=64, block_size=16, max_seqs=4, max_len=256, dtype=torch.float16,
                         device=dev)
    ws = cache.workspace(cache.max_seqs, 14)
    ws[:4096].view(torch.int32)[:4] = 1  # stale tickets
    cache.status.fill_(9)  # as a timed-out wait would have recorded
    with pytest.raises(RuntimeError, match="timed out"):
        cache.raise_device_errors()
    torch.cuda.synchronize()
    assert int(ws[:4096].view(torch.int32).abs().sum()) == 0
    assert int(cache.status.item()) == 0
