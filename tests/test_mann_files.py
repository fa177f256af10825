"""Index-file header parsing (no GPU): mans_mann_read_info on files written by
the test restatement of IndexSerializer (versions 1-3, 16 KiB and 4 KiB
pages), and the corruptFile checks of IndexSerializer.load /
MmapIndexLoader.load."""
import numpy as np
import pytest

import meltan_b200 as mb
from tests.mann_files import write_mann


@pytest.mark.parametrize("version,page", [(3, 16384), (3, 4096), (2, 0), (1, 0)])
def test_header_and_sections(tmp_path, version, page):
    v = np.arange(37 * 24, dtype=np.float32).reshape(37, 24)
    path = tmp_path / "x.mann"
    raw = write_mann(path, v, degree=5, metric=1, version=version, page_size=page or 16384,
                     entry_point=7)
    info = mb.mann_info(path)
    assert (info.version, info.count, info.degree, info.dim, info.metric) == (version, 37, 5, 24, 1)
    assert info.storage == 0 and info.entry_point == 7
    if version == 3:
        assert info.page_size == page and info.vector_offset == page
    got = np.frombuffer(raw[info.vector_offset:info.vector_offset + info.vector_bytes],
                        np.float32).reshape(37, 24)
    np.testing.assert_array_equal(got, v)
    assert raw[info.idmap_offset:info.idmap_offset + 1] == b"{"


def test_fp16_and_binary_storage_headers(tmp_path):
    v = np.linspace(-2, 2, 10 * 16, dtype=np.float32).reshape(10, 16)
    write_mann(tmp_path / "h.mann", v, storage=1)
    info = mb.mann_info(tmp_path / "h.mann")
    assert info.storage == 1 and info.vector_bytes == 10 * 16 * 2
    write_mann(tmp_path / "b.mann", np.zeros((10, 4), np.uint8), storage=2, metric=3)
    info = mb.mann_info(tmp_path / "b.mann")
    assert info.storage == 2 and info.dim == 32 and info.vector_bytes == 40


@pytest.mark.parametrize("damage", ["magic", "version", "truncate", "entry", "metric", "empty"])
def test_corrupt_files_are_rejected(tmp_path, damage):
    v = np.ones((9, 8), np.float32)
    path = tmp_path / "c.mann"
    raw = bytearray(write_mann(path, v, version=3, page_size=4096,
                               entry_point=8 if damage != "entry" else 9))
    if damage == "magic":
        raw[0:4] = b"NNAM"
    elif damage == "version":
        raw[4] = 9
    elif damage == "truncate":
        raw = raw[:-100]
    elif damage == "metric":
        raw[20] = 7
    elif damage == "empty":
        raw = raw[:10]
    path.write_bytes(bytes(raw))
    with pytest.raises(mb.CorruptFile):
        mb.mann_info(path)


@pytest.mark.gpu
@pytest.mark.parametrize("version,page,storage", [(3, 16384, 0), (3, 4096, 0), (2, 0, 0), (3, 16384, 1)])
def test_load_shards_and_search(ctx, tmp_path, version, page, storage):
    """loadReadOnly's vector section straight into device shards: every shard
    search merged equals the oracle on the whole file's rows (fp16 storage is
    widened exactly)."""
    import oracle as O
    v = O.lcg_vectors(5003, 48, 3)
    if storage == 1:
        v = v.astype(np.float16).astype(np.float32)
    q = O.lcg_vectors(4, 48, 4)
    path = tmp_path / "s.mann"
    write_mann(path, v, version=version, page_size=page or 16384, storage=storage)
    want = O.flat_search(v, q, 10, O.COSINE)
    pairs = [[] for _ in range(4)]
    for s in range(3):
        buf = mb.VectorBuffer.load_mann(ctx, path, s, 3)
        d, i, c = mb.FlatGPUSearch.batch_search_arrays(ctx, q, buf, 10, mb.Metric.cosine)
        for qi in range(4):
            pairs[qi] += [(float(d[qi, j]), int(i[qi, j])) for j in range(c[qi])]
        buf.close()
    for qi in range(4):
        got = sorted(pairs[qi])[:10]
        np.testing.assert_array_equal([g[1] for g in got], want[1][qi])
        np.testing.assert_array_equal(np.float32([g[0] for g in got]), want[0][qi])


@pytest.mark.gpu
def test_load_rejects_binary_storage(ctx, tmp_path):
    write_mann(tmp_path / "b.mann", np.zeros((10, 4), np.uint8), storage=2, metric=3)
    with pytest.raises(mb.SearchFailed):
        mb.VectorBuffer.load_mann(ctx, tmp_path / "b.mann")
