"""Encoder forward parity on the B200 against the CPU oracle (the reference's
scalar FP32 path restated) and the reference's own golden fixture.

Tolerance (the north star's bar, applied as is at every width): after L2
normalisation, cosine >= 0.99995 and max |gpu - reference| <= 1e-3, at every
Matryoshka dimension checked.  Token ids are passed through unchanged.

The reference's only trained-weight fixture (tiny_text, 3 layers of
trained-scale weights) amplifies the rounding of 11-bit-significand
products: with the default ("fast") precision its 8-dim embeddings land
within ~2e-3 of the reference, above the bar, and no single projection
carries the error (each alone adds 1e-4 to 9e-4).  The split precision
(svl_precision in svl_gpu.h: hi/lo-split TF32 products over every
projection, FP32 attention) meets the bar with ~1e-6 to spare, so the golden
tests run it; the fast path's envelope on that fixture is checked separately.
"""

import json
import os

import numpy as np
import pytest

import oracle
from svl import errors, synth
from svl.text import TextModel

pytestmark = pytest.mark.gpu

COS_MIN = 0.99995
MAX_ABS = 1e-3


def assert_embedding_close(gpu, ref, label, max_abs=MAX_ABS):
    """cosine >= 0.99995 and max abs <= 1e-3 (unscaled, at every width)."""
    gpu = np.asarray(gpu, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    cos = gpu @ ref / (np.linalg.norm(gpu) * np.linalg.norm(ref))
    err = np.abs(gpu - ref).max()
    assert cos >= COS_MIN and err <= max_abs, f"{label}: cosine {cos:.8f}, max abs {err:.2e} (bound {max_abs:.1e})"
    return cos, err


@pytest.fixture(scope="module")
def tiny(tiny_config, tiny_tensors):
    return TextModel(tiny_config, tiny_tensors, precision="split"), oracle.OracleModel(tiny_config, tiny_tensors)


def test_tiny_model_matches_the_golden_embeddings(tiny, tiny_golden):
    """tests/text_embeddings.rs:108-230: every case of the trained fixture,
    against its golden embedding and against the oracle, in split precision;
    every captured hidden state within 1e-4 of its row scale."""
    gpu, orc = tiny
    assert gpu.precision() == "split"
    for ci, case in enumerate(tiny_golden["cases"]):
        out = gpu.forward(case["input_ids"], capture_hidden=True)
        assert_embedding_close(out.normalized(), case["embedding"], f"case {ci} vs golden")
        ref = orc.forward(case["input_ids"], capture_hidden=True)
        _, e = assert_embedding_close(out.normalized(), ref["normalized"], f"case {ci} vs oracle", max_abs=2e-5)
        print(f"tiny_text split precision case {ci}: max abs vs oracle {e:.2e}")
        hs = np.stack(out.hidden_states())
        for layer in range(hs.shape[0]):
            d = np.abs(hs[layer] - ref["hidden_states"][layer]).max()
            scale = np.abs(ref["hidden_states"][layer]).max()
            assert d <= 1e-4 * scale + 1e-7, f"case {ci} layer {layer}: {d} vs scale {scale}"
        t = out.embedding(4)
        assert abs(float(t @ t) - 1.0) <= 1e-4


def test_tiny_model_fast_precision_envelope(tiny_config, tiny_tensors, tiny_golden):
    """The default precision on the trained fixture: cosine >= 0.99995 holds,
    the element error stays within 4e-3 (11-bit products through 3 layers of
    trained-scale weights; measured ~2e-3) -- the reason split precision
    exists."""
    fast = TextModel(tiny_config, tiny_tensors, precision="fast")
    assert fast.precision() == "fast"
    errs = []
    for ci, case in enumerate(tiny_golden["cases"]):
        out = fast.forward(case["input_ids"]).normalized()
        errs.append(assert_embedding_close(out, case["embedding"], f"fast case {ci}", max_abs=4e-3)[1])
    print(f"tiny_text fast precision: max abs per case {['%.2e' % e for e in errs]}")


def test_tiny_model_batch_equals_single_calls(tiny, tiny_golden):
    gpu, _ = tiny
    seqs = [c["input_ids"] for c in tiny_golden["cases"]]
    batch = gpu.forward_batch(seqs)["normalized"]
    for i, s in enumerate(seqs):
        single = gpu.forward(s).normalized()
        assert_embedding_close(batch[i], single, f"seq {i}")


def test_forward_is_deterministic(tiny):
    gpu, _ = tiny
    a = gpu.embed_ids([1, 5, 7, 9, 2], 8)
    b = gpu.embed_ids([1, 5, 7, 9, 2], 8)
    assert np.array_equal(a, b)


def test_concurrent_calls_from_threads_match_sequential_calls(small_manifest):
    """tests/text_embeddings.rs:432-457: one model called from several host
    threads at once (ctypes releases the GIL, so the C calls overlap and the
    handle's mutex serialises them) returns what sequential calls return, bit
    for bit."""
    import threading

    cfg, gpu, _ = small_manifest
    rng = np.random.default_rng(21)
    seqs = [rng.integers(2, cfg.vocab_size, n).astype(np.uint32) for n in (5, 40, 131, 300)]
    want = [gpu.embed_ids(s, 768) for s in seqs]
    got = [None] * 6
    failures = []

    def run(t):
        try:
            got[t] = [gpu.embed_ids(seqs[(t + j) % len(seqs)], 768) for j in range(len(seqs))]
        except Exception as e:  # reported below, on the main thread
            failures.append(repr(e))

    threads = [threading.Thread(target=run, args=(t,)) for t in range(len(got))]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not failures, failures
    assert not any(th.is_alive() for th in threads)
    for t, out in enumerate(got):
        for j, e in enumerate(out):
            assert np.array_equal(e, want[(t + j) % len(seqs)]), (t, j)


def test_engine_embed_tokens_is_the_model_call(small_manifest):
    """api/engine.rs:222-234: after its own checks the engine returns the
    model's embedding for the same ids and dimension."""
    from svl.engine import Engine

    cfg, gpu, _ = small_manifest
    ids = np.random.default_rng(5).integers(2, cfg.vocab_size, 77).astype(np.uint32)
    for dim in Engine(gpu).matryoshka_dimensions():
        assert np.array_equal(Engine(gpu).embed_tokens(ids, dim), gpu.embed_ids(ids, dim))


def test_invalid_inputs_raise_the_reference_errors(tiny, tiny_config):
    gpu, _ = tiny
    with pytest.raises(errors.CorruptError):
        gpu.forward([])
    with pytest.raises(errors.CorruptError):
        gpu.forward([1, tiny_config.vocab_size])
    with pytest.raises(errors.LimitExceededError):
        gpu.forward([1] * (tiny_config.max_position_embeddings + 1))
    with pytest.raises(errors.InternalError):
        gpu.embed_ids([1, 2], 0)
    with pytest.raises(errors.InternalError):
        gpu.embed_ids([1, 2], tiny_config.embedding_dim + 1)
    # the model stays usable after rejected calls
    assert np.isfinite(gpu.embed_ids([1, 2], 4)).all()


def test_forward_with_features_matches_the_oracle(tiny, tiny_config):
    gpu, orc = tiny
    rng = np.random.default_rng(3)
    ids = [1, 5, 7, 9, 11, 2]
    feats = rng.standard_normal((2, tiny_config.hidden_size)).astype(np.float32)
    out = gpu.forward_with_features(ids, feats, 2, 2)
    ref = orc.forward(ids, features=feats, feature_start=2)
    assert_embedding_close(out.normalized(), ref["normalized"], "features")


def _text_model(cfg, w, attention):
    """A model whose attention and GEMM operands are FP16 (the default) or,
    with SVL_ATTENTION_TF32=1 and SVL_GEMM_TF32=1 set while it is created,
    FP32 for the TF32 kernels; "f16_separate_qkv" runs the q/k/v norms and
    RoPE as a separate kernel instead of the QKV GEMM's epilogue;
    "f16_unfused_rows" runs the o / down projections and the per-layer-input
    block as separate GEMMs and residual kernels (SVL_ROW_FUSED=0); "split" is the split
    precision (svl_model_create_ex)."""
    if attention == "split":
        return TextModel(cfg, w, precision="split")
    if attention == "tf32":
        os.environ["SVL_ATTENTION_TF32"] = "1"
        os.environ["SVL_GEMM_TF32"] = "1"
    if attention == "f16_separate_qkv":
        os.environ["SVL_QKV_EPILOGUE"] = "0"
    if attention == "f16_unfused_rows":
        os.environ["SVL_ROW_FUSED"] = "0"
    try:
        return TextModel(cfg, w)
    finally:
        for k in ("SVL_ATTENTION_TF32", "SVL_GEMM_TF32", "SVL_QKV_EPILOGUE", "SVL_ROW_FUSED"):
            os.environ.pop(k, None)


@pytest.fixture(scope="module")
def small_manifest():
    cfg = synth.manifest_config(num_layers=2, vocab_size=4096)
    w = synth.random_weights(cfg, seed=11)
    return cfg, TextModel(cfg, w), oracle.OracleModel(cfg, w)


@pytest.mark.parametrize("attention", ["f16", "tf32", "f16_separate_qkv", "f16_unfused_rows", "split"])
def test_manifest_width_batch_matches_the_oracle(small_manifest, attention):
    """Manifest widths (hidden 512, heads 4, kv 2x256 sliding / 1x512 full, FFN
    2048, PLE 512, output 768) on a ragged batch, including a sequence longer
    than the 512-token window."""
    cfg, gpu, orc = small_manifest
    if attention != "f16":
        gpu = _text_model(cfg, synth.random_weights(cfg, seed=11), attention)
    rng = np.random.default_rng(9)
    lens = [1, 2, 31, 130, 600]
    seqs = [rng.integers(2, cfg.vocab_size, size=n).astype(np.uint32) for n in lens]
    for dim in (768, 256):
        got = gpu.embed_batch(seqs, dim)
        for i, s in enumerate(seqs):
            ref = oracle.truncate_and_normalize(orc.forward(s)["normalized"], dim)
            assert_embedding_close(got[i], ref, f"len {lens[i]} dim {dim}")


@pytest.mark.parametrize("attention", ["f16", "tf32", "split"])
def test_unit_scale_stress_model(small_manifest, attention):
    """Norm weights ~ 1 + N(0, 0.02): unit-scale activations and large
    attention logits (scale 1.0 on RMS-normed q, k)."""
    cfg, _, _ = small_manifest
    w = synth.random_weights(cfg, seed=12, unit_norms=True)
    gpu, orc = _text_model(cfg, w, attention), oracle.OracleModel(cfg, w)
    rng = np.random.default_rng(4)
    seqs = [rng.integers(2, cfg.vocab_size, size=n).astype(np.uint32) for n in (17, 200)]
    got = gpu.embed_batch(seqs, 768)
    for i, s in enumerate(seqs):
        assert_embedding_close(got[i], orc.forward(s)["normalized"], f"stress seq {i}")


def test_split_batch_is_bitwise_equal_to_unsplit_calls(small_manifest):
    """A batch of >= 8192 tokens runs as two halves on two streams; every
    sequence's arithmetic is independent of the grouping, so the embeddings
    must equal, bit for bit, those of smaller (single-stream) calls."""
    cfg, gpu, orc = small_manifest
    rng = np.random.default_rng(17)
    lens = rng.integers(300, 600, size=22)
    assert lens.sum() >= 8192
    seqs = [rng.integers(2, cfg.vocab_size, size=int(n)).astype(np.uint32) for n in lens]
    whole = gpu.embed_batch(seqs, 768)
    parts = np.concatenate([gpu.embed_batch(seqs[i:i + 5], 768) for i in range(0, len(seqs), 5)])
    assert np.array_equal(whole, parts)
    assert_embedding_close(whole[13], orc.forward(seqs[13])["normalized"], "split batch, sequence 13")


def test_device_entry_point_matches_host_entry_point(small_manifest):
    import torch

    cfg, gpu, _ = small_manifest
    rng = np.random.default_rng(1)
    seqs = [rng.integers(2, cfg.vocab_size, size=n).astype(np.uint32) for n in (40, 64, 3)]
    from svl.text import pack

    ids, cu = pack(seqs)
    host = gpu.embed_packed(ids, cu, 256)
    d_ids = torch.from_numpy(ids.astype(np.int32)).cuda()
    d_out = torch.empty((len(seqs), 256), device="cuda")
    torch.cuda.synchronize()
    gpu.embed_batch_device(d_ids.data_ptr(), cu, 256, d_out.data_ptr())
    gpu.check()
    assert np.array_equal(d_out.cpu().numpy(), host)


@pytest.mark.parametrize("own_stream", [False, True])
def test_back_to_back_device_calls_match_synchronous_calls(small_manifest, own_stream):
    """Device-entry calls on four different batches, issued back to back
    (twice over) with no synchronisation between them -- each batch is at
    least 8192 tokens, so each runs as two half-batches on two streams whose
    kernels use programmatic dependent launch.  Every output must equal, bit
    for bit, the synchronous host-entry result of its own batch: no call may
    read an earlier call's inputs, schedules or activations, nor a later
    call overwrite them early.  Run on a caller stream and on the model's
    own stream (a NULL stream handle)."""
    import torch

    from svl.text import pack

    cfg, gpu, _ = small_manifest
    rng = np.random.default_rng(23)
    batches = []
    for b in range(4):
        lens = rng.integers(60 + 40 * b, 600, size=24 + 4 * b)
        lens[0] = 8192 - int(lens[1:].sum()) if lens.sum() < 8192 else lens[0]
        seqs = [rng.integers(2, cfg.vocab_size, size=int(n)).astype(np.uint32) for n in lens]
        ids, cu = pack(seqs)
        assert cu[-1] >= 8192
        batches.append((ids, cu, gpu.embed_packed(ids, cu, 768)))
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        d_in = [torch.from_numpy(ids.astype(np.int32)).cuda() for ids, _, _ in batches]
        d_out = [torch.full((cu.size - 1, 768), float("nan"), device="cuda") for _, cu, _ in batches]
    torch.cuda.synchronize()
    handle = None if own_stream else stream.cuda_stream
    for _ in range(2):
        for (_, cu, _), di, do in zip(batches, d_in, d_out):
            gpu.embed_batch_device(di.data_ptr(), cu, 768, do.data_ptr(), handle)
    torch.cuda.synchronize()
    gpu.check()
    for b, ((_, _, want), do) in enumerate(zip(batches, d_out)):
        assert np.array_equal(do.cpu().numpy(), want), f"batch {b}"


def test_full_model_config1_matches_the_oracle():
    """the 24-layer manifest model, random N(0, 0.02)
    weights (seed 1234), one 32-token SearchQuery sequence."""
    cfg = synth.manifest_config()
    w = synth.random_weights(cfg, seed=1234)
    gpu = TextModel(cfg, w)
    orc = oracle.OracleModel(cfg, w)
    ids = synth.config1_ids()
    ref = orc.forward(ids)["normalized"]
    out = gpu.forward(ids)
    for dim in (768, 512, 256, 128):
        assert_embedding_close(out.embedding(dim), oracle.truncate_and_normalize(ref, dim), f"config1 dim {dim}")


def test_text_embedder_runs_the_tokenizer_then_the_encoder():
    """TextEmbedder::embed (text.rs:616-626): prompt prefix, the frozen
    tokenizer (the reduced tokenizer.json, on golden-corpus texts it
    reproduces) with <bos> / <eos>, then the encoder; the embeddings match the
    oracle's on the same ids (a 2-layer model at the full 262,144-token
    vocabulary, so the real token ids index the embedding tables)."""
    from conftest import GOLDEN
    from svl.prompt import Prompt, apply
    from svl.text import TextEmbedder
    from svl.tokenizer import Tokenizer

    cfg = synth.manifest_config(num_layers=2)
    w = synth.random_weights(cfg, seed=5)
    tok = Tokenizer.load(GOLDEN / "tokenizer" / "mini_tokenizer.json")
    embedder = TextEmbedder(TextModel(cfg, w), tok)
    orc = oracle.OracleModel(cfg, w)
    corpus = {c["name"]: c for c in json.loads((GOLDEN / "tokenizer" / "golden.json").read_text())["cases"]}
    texts = [corpus[n]["text"] for n in ("english_sentence", "french_diacritics", "emoji", "long_text")]
    for prompt in (Prompt.Document, Prompt.SearchQuery):
        got = embedder.embed_many(texts, prompt, 768)
        for i, text in enumerate(texts):
            ids = embedder.token_ids(text, prompt)
            assert list(ids) == tok.encode(apply(prompt, text), True)
            assert_embedding_close(got[i], orc.forward(ids)["normalized"], f"{prompt.name} text {i}")
        one = embedder.embed(texts[0], prompt, 256)
        assert np.array_equal(one, embedder.model().embed_ids(embedder.token_ids(texts[0], prompt), 256))
