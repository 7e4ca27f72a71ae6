"""Cold chunks as NPZ files in the reference's format (storage.py:113-151), on the CPU.

tests/golden/ref_chunks/ holds chunk files written by the reference cache
itself (tests/golden/make_golden.py, case chunk_files): a 20-token chunk made
by merging a whole 16-token piece onto a 4-token partial chunk, and the chunk
after it.  The B200 build's reader and writer (apple_b200/chunk_io.py) must
round-trip them array for array, and the oracle's cold tier must hold the same
chunks with the same codes.
"""
import numpy as np
import pytest

from oracle import restate as R
from tests.conftest import GOLDEN

REF = GOLDEN / "ref_chunks"


def _ref_files():
    idx = dict(np.load(REF / "index.npz"))
    return idx, [REF / f"layer0_chunk{int(c)}.npz" for c in idx["chunk_ids"]]


@pytest.mark.parametrize("which", [0, 1])
def test_reader_and_writer_round_trip_reference_files(tmp_path, which):
    from apple_b200.chunk_io import compressed_tensor_from_loaded, load_compressed_chunk, save_compressed_chunk
    _, files = _ref_files()
    src = files[which]
    loaded = load_compressed_chunk(src)
    keys = compressed_tensor_from_loaded(loaded, "key", num_rvq_layers=1)
    values = compressed_tensor_from_loaded(loaded, "value", num_rvq_layers=1)
    assert keys.num_tokens == int(loaded["num_tokens"][0]) and keys.num_heads == int(loaded["num_heads"][0])
    out = tmp_path / src.name
    save_compressed_chunk(out, keys, values)
    a, b = np.load(src), np.load(out)
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)


def test_oracle_cold_tier_matches_reference_chunk_files():
    idx, files = _ref_files()
    cfg = R.OracleConfig(hidden_dim=256, num_heads=4, head_dim=64, num_subspaces=16, subspace_dim=4, num_rvq_layers=1,
                         rvq_codebook_size=256, rvq_sparsity_threshold=0.4, hot_capacity=16, warm_capacity=24,
                         block_size_seq=16)
    cache = R.OracleCache(cfg, R.Quantizer(idx["pq_codebooks"], idx["rvq_codebooks"], 0.4))
    s = int(idx["update_split"])
    cache.update(idx["keys"][None, :s], idx["values"][None, :s])
    cache.update(idx["keys"][None, s:], idx["values"][None, s:])
    assert [m["chunk_id"] for m in cache.cold] == list(idx["chunk_ids"])
    assert [[m["start_token"], m["end_token"]] for m in cache.cold] == idx["chunk_bounds"].tolist()
    for meta, path in zip(cache.cold, files):
        f = np.load(path)
        for prefix, codes in (("key", meta["k"][0]), ("value", meta["v"][0])):
            np.testing.assert_array_equal(codes.pq, f[f"{prefix}_pq_codes"])
            np.testing.assert_array_equal(codes.mask, f[f"{prefix}_rvq_mask"])
            flat = codes.mask.reshape(-1)
            np.testing.assert_array_equal(np.flatnonzero(flat), f[f"{prefix}_rvq_offsets"])
            np.testing.assert_array_equal(codes.rvq.reshape(-1, 1)[flat], f[f"{prefix}_rvq_codes"])
