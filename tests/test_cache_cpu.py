"""Host logic of the decode path that needs no GPU: the KV cache store's views and growth
policy, and how the indexer pass groups query rows into chunks (whole sequences per launch
when a sequence's rows fit)."""

import torch


def test_cache_store_views_share_its_buffers():
    from gsa_b200.attention import KVCacheStore, _grown_capacity

    st = KVCacheStore(3, 40, 2, 16, 8, torch.float32, "cpu")
    c = st.view(25)
    assert c[0].shape == (3, 25, 2, 16) and c[1].shape == (3, 25, 2, 16) and c.indexer_keys.shape == (3, 25, 8)
    assert c.store is st and c.capacity == 40
    assert c[0].data_ptr() == st.kv.data_ptr() and c[1].data_ptr() == st.kv[:, :, 1].data_ptr()
    # k and v of a token are adjacent: the interleaved layout the sparse SDPA copies in one piece
    assert c[0].stride(1) == 2 * 2 * 16 and c[1].data_ptr() - c[0].data_ptr() == 2 * 16 * 4
    assert c[0].stride(0) == 40 * 2 * 2 * 16
    assert st.fits(3, 40, torch.float32, torch.device("cpu")) and not st.fits(3, 41, torch.float32, torch.device("cpu"))
    assert not st.fits(2, 10, torch.float32, torch.device("cpu"))
    for n in (1, 255, 256, 1000, 65537):
        cap = _grown_capacity(n)
        assert cap % 256 == 0 and cap >= n + 256 and cap >= n * 5 // 4


def test_indexer_chunking_groups_whole_sequences():
    from gsa_b200 import ops

    ld = lambda n: (n + 3) // 4 * 4  # noqa: E731
    cap_rows = ops.SCORE_CHUNK_BYTES // (4 * ld(65537))
    # decode: 64 sequences of one row share one chunk
    assert ops._chunking(64, 1, 65537, None) == (64, 1)
    # prefill of one long sequence: row chunks of that sequence
    rows, n = ops._chunking(1, 131072, 131072, None)
    assert rows == ops.SCORE_CHUNK_BYTES // (4 * 131072) and n == 131072 // rows
    # several sequences that fit together
    assert ops._chunking(2, 8192, 8192, None) == (16384, 1)
    assert ops._chunking(300, 1000, 65537, None) == (cap_rows // 1000 * 1000, -(-300 // (cap_rows // 1000)))
    # explicit chunk rows
    assert ops._chunking(3, 1100, 1100, 500) == (500, 9)
    assert ops._chunking(5, 2, 100, 5) == (5, 3)
