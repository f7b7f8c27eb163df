"""Row gather (the embedding lookup, yllang::Index, src/layers/index.cu:93-146)
on the GPU, byte for byte against the CPU oracle: every row-shape family,
int32 and int64 indices, strided tables and outputs, misaligned rows (generic
kernel), out-of-range indices (zero rows, -1 silent, others flagged), the
Qwen3-0.6B embedding table shape, and the C++ front end's Index."""
import numpy as np
import pytest
import torch

import yllang_b200 as yl
from _kvutil import host_bytes, random_bytes
from oracle import kvpath as orc

pytestmark = pytest.mark.gpu


def _check(table, idx, out=None, err=None):
    got = yl.gather_rows(idx, table, out=out, error_word=err)
    torch.cuda.synchronize()
    want, bits = orc.gather(idx.cpu().numpy(), host_bytes(table).reshape(table.shape[0], -1))
    assert np.array_equal(host_bytes(got).reshape(got.shape[0], -1), want)
    return got, bits


@pytest.mark.parametrize("row_bytes", [16, 48, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 12288])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_gather_row_sizes(cuda, row_bytes, idx_dtype):
    V = 3000
    table = random_bytes((V, row_bytes), row_bytes).to(cuda)
    g = torch.Generator().manual_seed(row_bytes + 1)
    for n in (1, 7, 333, 5000):
        idx = torch.randint(0, V, (n,), generator=g).to(idx_dtype).to(cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        _, bits = _check(table, idx, err=err)
        assert bits == 0 and int(err.item()) == 0


@pytest.mark.parametrize("row_bytes,offset", [(6, 0), (2, 0), (40, 8), (256, 4), (1000, 0), (4096, 2)])
def test_gather_generic_alignments(cuda, row_bytes, offset):
    V, n = 500, 777
    flat = random_bytes((V * (row_bytes + 16) + 64,), 3).to(cuda)
    stride = row_bytes + 16 if offset else row_bytes
    table = flat[offset:offset + V * stride].view(V, stride)[:, :row_bytes]
    idx = torch.randint(0, V, (n,), generator=torch.Generator().manual_seed(4)).to(cuda)
    _check(table, idx)


def test_gather_strided_table_and_out(cuda):
    V, E = 2048, 1024
    big = torch.randn(V, E + 64, device=cuda).to(torch.bfloat16)
    table = big[:, 32:32 + E]
    out_buf = torch.full((600, E + 128), 7, dtype=torch.bfloat16, device=cuda)
    out = out_buf[:, 64:64 + E]
    idx = torch.randint(0, V, (600,), generator=torch.Generator().manual_seed(5)).to(cuda)
    got = yl.gather_rows(idx, table, out=out)
    torch.cuda.synchronize()
    assert got.data_ptr() == out.data_ptr()
    assert torch.equal(out, table[idx.long()])
    assert bool((out_buf[:, :64] == 7).all()) and bool((out_buf[:, 64 + E:] == 7).all())


def test_gather_out_of_range_rows(cuda):
    V, E = 100, 256
    table = random_bytes((V, E), 9).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _, bits = _check(table, torch.tensor([3, -1, 99, -1], dtype=torch.int64, device=cuda), err=err)
    assert bits == 0 and int(err.item()) == 0
    for bad in ([5, 100, 7], [-2, 0], [2**40, 1]):
        err.zero_()
        got, bits = _check(table, torch.tensor(bad, dtype=torch.int64, device=cuda), err=err)
        assert bits == orc.INDEX_RANGE and int(err.item()) == yl.DEVERR_INDEX_RANGE
    err.zero_()
    got, bits = _check(table, torch.tensor([1, 100, -3], dtype=torch.int32, device=cuda), err=err)
    assert int(err.item()) == yl.DEVERR_INDEX_RANGE and int(got[1:].abs().sum()) == 0


def test_gather_empty_and_errors(cuda):
    table = torch.zeros(10, 64, dtype=torch.bfloat16, device=cuda)
    out = yl.gather_rows(torch.zeros(0, dtype=torch.int32, device=cuda), table)
    assert out.shape == (0, 64)
    with pytest.raises(yl.PanicError):
        yl.gather_rows(torch.zeros(4, dtype=torch.int16, device=cuda), table)
    with pytest.raises(yl.PanicError):
        yl.gather_rows(torch.zeros(4, dtype=torch.int32, device=cuda), table,
                       out=torch.empty(4, 32, dtype=torch.bfloat16, device=cuda))


def test_gather_qwen3_embedding_shape(cuda):
    """Qwen3-0.6B token embedding: 151936 x 1024 bf16, 4096 tokens (prefill)
    and 256 tokens (decode)."""
    V, E = 151936, 1024
    table = torch.randn(V, E, device=cuda, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(11)
    for n in (256, 4096):
        idx = torch.randint(0, V, (n,), generator=g, dtype=torch.int32).to(cuda)
        got = yl.gather_rows(idx, table)
        torch.cuda.synchronize()
        assert torch.equal(got, table[idx.long()])


def test_cpp_index_front_end(cuda):
    C = yl.load_extension()
    V, E = 4000, 768
    w = torch.randn(V, E, device=cuda).to(torch.bfloat16)
    idx = torch.randint(0, V, (1000,), generator=torch.Generator().manual_seed(12)).to(cuda)
    dst = torch.empty(1000, E, dtype=torch.bfloat16, device=cuda)
    C.Index(idx, w, dst)
    torch.cuda.synchronize()
    assert torch.equal(dst, w[idx])
    with pytest.raises(C.PanicError):
        C.Index(idx.to(torch.int16), w, dst)
    with pytest.raises(C.PanicError):
        C.Index(idx, w, dst.float())
