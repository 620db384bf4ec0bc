"""The centroid index and the indexing job: file round trip with reference
samples for some adapters only, replacement in place, independent
snapshots, foreign files read as absent, checkpoints that only resume the
same job, and fingerprints that separate every field."""
import numpy as np

from deltaserve_vllm_b200.adapters.routing.index import CentroidIndex, Indexer, fingerprint, l2_normalize


def test_index_round_trip_replace_and_snapshot(tmp_path):
    rng = np.random.default_rng(0)
    idx = CentroidIndex("enc", "query: ", 128)
    for n in "abc":
        idx.add(n, rng.normal(size=8), refs=rng.normal(size=(3, 8)) if n != "b" else None)
    snap = idx.snapshot()
    idx.add("a", np.ones(8))                                  # replaced in place, without references now
    assert idx.names == ["a", "b", "c"] and set(idx.refs) == {"c"}
    np.testing.assert_allclose(idx.matrix[0], l2_normalize(np.ones(8)), rtol=1e-6)
    assert not np.allclose(snap.matrix[0], idx.matrix[0])     # the snapshot kept the old centroid
    path = str(tmp_path / "i.npz")
    idx.save(path)
    back = CentroidIndex.load(path)
    assert (back.encoder, back.prefix, back.max_tokens) == ("enc", "query: ", 128)
    assert back.names == idx.names and set(back.refs) == {"c"}
    np.testing.assert_allclose(back.matrix, idx.matrix)
    np.testing.assert_allclose(back.refs["c"], idx.refs["c"])
    q = rng.normal(size=8)
    np.testing.assert_allclose(back.scores(q), idx.matrix @ l2_normalize(q), rtol=1e-5)
    assert idx.remove("b") and not idx.remove("b") and idx.names == ["a", "c"] and idx.matrix.shape == (2, 8)
    import pytest
    with pytest.raises(ValueError, match="dim"):
        idx.add("a", np.ones(5))                               # even when replacing an entry
    np.savez(str(tmp_path / "other.npz"), meta=np.array("x"))
    assert CentroidIndex.load_or_none(str(tmp_path / "other.npz")) is None
    assert CentroidIndex.load_or_none(str(tmp_path / "missing.npz")) is None


def test_checkpoint_resumes_only_the_same_job(tmp_path):
    rng = np.random.default_rng(2)
    texts = [f"t{i}" for i in range(20)]
    emb = rng.normal(size=(20, 4))
    ck = str(tmp_path / "ck.npz")
    ix = Indexer(texts, "fp", ck, reference_samples=4)
    assert ix.commit(0, emb[:9])
    assert Indexer(texts, "fp", ck, reference_samples=4).resumed_from == 9
    assert Indexer(texts, "fp", ck, reference_samples=3).resumed_from == 0     # another reference setting
    assert Indexer(texts[:-1], "fp", ck, reference_samples=4).resumed_from == 0  # another sample list
    ix2 = Indexer(texts, "fp", ck, reference_samples=4)
    assert not ix2.commit(8, emb[8:12])                       # not the current chunk
    while not ix2.done:
        s, chunk = ix2.next_chunk(5)
        assert ix2.commit(s, emb[s:s + len(chunk)])
    refs = ix2.references()
    pos = [0, 6, 13, 19]                                      # evenly spread over 20 samples
    np.testing.assert_allclose(refs, l2_normalize(emb[pos]).astype(np.float32), rtol=1e-6)
    np.testing.assert_allclose(ix2.centroid(), l2_normalize(l2_normalize(emb).mean(0)), rtol=1e-5, atol=1e-6)


def test_fingerprint_separates_fields():
    t = ["ab", "c"]
    base = fingerprint(t, "enc", "p", 64)
    assert base == fingerprint(list(t), "enc", "p", 64)
    assert len({base, fingerprint(["a", "bc"], "enc", "p", 64), fingerprint(t, "enc2", "p", 64),
                fingerprint(t, "enc", "q", 64), fingerprint(t, "enc", "p", 65), fingerprint(t[:1], "enc", "p", 64)}) == 6
