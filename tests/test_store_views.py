"""Batch-slice views of the cache structs (host arithmetic only, no kernel
launch): ``Int4KVStore.struct(b0=...)`` and ``DenseKV.struct(b0=...)`` describe
sequences [b0, batch) so that a launch over a batch slice reads the same pages,
page-table rows, lengths and dense rows as the full-batch launch does for those
sequences; ``SeqSplitDecoder`` refuses slice counts outside [1, batch]."""
import pytest
import torch

from hetero_kvcache_optimizer_b200 import kvstore as kv


@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("b0", [0, 1, 2])
def test_int4_store_view(paged, b0):
    B, H = 3, 2
    st = kv.Int4KVStore(B, H, 600, fmt="fp16min", group=32, num_pages=40 if paged else None, device="cpu")
    full, view = st.struct(), st.struct(b0=b0)
    skip = b0 * H * st.max_pages
    assert view.lengths == full.lengths + 4 * b0
    assert (view.format, view.group, view.page_tokens, view.max_pages, view.page_stride) == \
        (full.format, full.group, full.page_tokens, full.max_pages, full.page_stride)
    if paged:
        # same pool, table rows of unit b0*H on
        assert view.pages == full.pages and view.num_pages == full.num_pages
        assert view.page_table == st.page_table[b0 * H].data_ptr()
    else:
        # unit u of the view is unit b0*H + u of the store: its page 0 is page skip
        assert view.page_table is None and full.page_table is None
        assert view.pages == full.pages + skip * st.page_bytes
        assert view.num_pages == full.num_pages - skip


@pytest.mark.parametrize("b0", [0, 2])
def test_dense_view(b0):
    d = kv.DenseKV(3, 2, 40, dtype=torch.bfloat16, device="cpu")
    full, view = d.struct(), d.struct(b0=b0)
    assert view.k == d.k[b0].data_ptr() and view.v == d.v[b0].data_ptr()
    assert view.lengths == full.lengths + 4 * b0
    assert (view.stride_b, view.stride_h, view.stride_t, view.capacity, view.dtype) == \
        (full.stride_b, full.stride_h, full.stride_t, full.capacity, full.dtype)


def test_view_outside_batch_refused():
    st = kv.Int4KVStore(2, 2, 256, fmt="fp16min", group=32, device="cpu")
    d = kv.DenseKV(2, 2, 8, device="cpu")
    for bad in (-1, 2):
        with pytest.raises(ValueError):
            st.struct(b0=bad)
        with pytest.raises(ValueError):
            d.struct(b0=bad)


def test_decoder_slice_count_checked():
    from hetero_kvcache_optimizer_b200.seqsplit import SeqSplitDecoder
    for chunks in (0, 5):
        with pytest.raises(ValueError):
            SeqSplitDecoder([None], [None], 4, 8, device="cpu", chunks=chunks)
