"""Document ingest into the device index on the B200 (svl_ingest_batch,
VectorIndex.ingest): the chunk embedding of Store::put_document
(src/storage/store.rs:524), Chunk::new's f64 normalisation
(src/storage/model.rs:546-581) and the index append, with the embeddings
kept on the GPU.  Its result must be the host path's exactly (embed to host
buffers, then append): the same stored rows, so identical search results with
bit-identical f64 scores; the device-pointer append is checked the same way."""

from __future__ import annotations

import numpy as np
import pytest

from svl import errors, synth
from svl.index import VectorIndex
from svl.text import TextModel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    cfg = synth.manifest_config(num_layers=2, vocab_size=4096)
    return TextModel(cfg, synth.random_weights(cfg, seed=21))


def _seqs(seed, n, vocab=4096):
    rng = np.random.default_rng(seed)
    return [rng.integers(2, vocab, size=int(k)).astype(np.uint32) for k in rng.integers(3, 260, size=n)]


def _same_results(a: VectorIndex, b: VectorIndex, queries, k=10):
    ra, rb = a.search(queries, k), b.search(queries, k)
    for x, y in zip(ra, rb):
        assert np.array_equal(np.asarray(x), np.asarray(y))


@pytest.mark.parametrize("dim", [768, 256])
def test_ingest_equals_embedding_on_the_host_then_appending(model, dim):
    docs = _seqs(1, 48)
    chunk_ids = np.arange(1000, 1048, dtype=np.uint64)[::-1].copy()
    ingested = VectorIndex(dim, 128)
    ingested.ingest(model, docs[:20], chunk_ids[:20])
    ingested.ingest(model, docs[20:], chunk_ids[20:])  # two calls append in order
    host = VectorIndex(dim, 128)
    host.append(model.embed_batch(docs, dim), chunk_ids)
    assert len(ingested) == len(host) == 48
    queries = model.embed_batch(_seqs(2, 6), dim)
    queries = np.concatenate([queries, host_rows_probe(model, docs[:2], dim)])
    _same_results(ingested, host, queries)


def host_rows_probe(model, docs, dim):
    # stored documents as queries: their own rows must come back first with score 1
    return model.embed_batch(docs, dim)


def test_device_pointer_append_equals_the_host_append(model):
    import torch

    from svl.text import pack

    docs = _seqs(3, 24)
    chunk_ids = np.arange(24, dtype=np.uint64) * 7
    ids, cu = pack(docs)
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    d_out = torch.empty((len(docs), 768), device="cuda")
    d_chunk = torch.from_numpy(chunk_ids.view(np.int64)).cuda()
    model.embed_batch_device(d_ids.data_ptr(), cu, 768, d_out.data_ptr())
    model.check()
    dev = VectorIndex(768, 64)
    torch.cuda.synchronize()
    dev.append_device(d_out.data_ptr(), d_chunk.data_ptr(), len(docs))
    dev.check()
    host = VectorIndex(768, 64)
    host.append(d_out.cpu().numpy(), chunk_ids)
    _same_results(dev, host, model.embed_batch(_seqs(4, 5), 768))


def test_ingest_rejects_bad_batches_before_touching_the_index(model):
    idx = VectorIndex(768, 8)
    with pytest.raises(errors.LimitExceededError, match="capacity"):
        idx.ingest(model, _seqs(5, 9), np.arange(9))
    assert len(idx) == 0
    bad = _seqs(6, 3)
    bad[1][0] = 4096  # outside the vocabulary: text.rs:188-218 -> Corrupt, nothing appended
    with pytest.raises(errors.CorruptError):
        idx.ingest(model, bad, np.arange(3))
    assert len(idx) == 0
    with pytest.raises(errors.UsageError):
        VectorIndex(1024, 8).ingest(model, _seqs(7, 2), np.arange(2))  # wider than the model's 768
    with pytest.raises(errors.UsageError):
        idx.ingest(model, _seqs(8, 2), np.arange(3))
    idx.ingest(model, _seqs(9, 8), np.arange(8))
    assert len(idx) == 8
