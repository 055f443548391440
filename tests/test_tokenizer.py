"""The BPE tokenizer front end (include/svl_tokenizer.h, src/model/tokenizer.rs)
and the prompt prefixes (src/model/prompt.rs), on the CPU.

Parity is pinned to the reference's golden corpus: token ids and decoded text
that the official tokenizers 0.23.3 library produced with the frozen
tokenizer.json, replayed here with the reduced tokenizer that reproduces it
(tests/tokenizer.rs:61-100), plus the unit cases of tokenizer.rs:860-1078 and
prompt.rs:98-151.  Beyond the corpus the product's heap-based merge loop is
compared with a literal restatement of the reference's quadratic loop
(oracle/bpe_ref.py) on seeded random text.
"""

from __future__ import annotations

import json
import random

import pytest

from conftest import GOLDEN
from oracle.bpe_ref import RefTokenizer
from svl import errors, prompt
from svl.tokenizer import MAX_INPUT_BYTES, Tokenizer

MINI_PATH = GOLDEN / "tokenizer" / "mini_tokenizer.json"
MINI = MINI_PATH.read_text(encoding="utf-8")
CORPUS = json.loads((GOLDEN / "tokenizer" / "golden.json").read_text(encoding="utf-8"))


@pytest.fixture(scope="module")
def mini():
    return Tokenizer.from_json_str(MINI)


@pytest.fixture(scope="module")
def ref():
    return RefTokenizer(MINI)


# ------------------------------------------------------------ golden corpus
@pytest.mark.parametrize("case", CORPUS["cases"], ids=[c["name"] for c in CORPUS["cases"]])
def test_golden_corpus(mini, case):
    """tests/tokenizer.rs:61-100: ids without and with <bos>/<eos>, and the
    decoded text (special tokens skipped) of both id lists."""
    assert mini.encode(case["text"], False) == case["ids"]
    assert mini.encode(case["text"], True) == case["ids_with_special"]
    assert mini.decode(case["ids"], True) == case["decoded"]
    assert mini.decode(case["ids_with_special"], True) == case["decoded"]


def test_the_restatement_reproduces_the_golden_corpus(ref):
    """Pins the oracle: the literal restatement gives the official ids too."""
    for case in CORPUS["cases"]:
        assert ref.encode(case["text"], False) == case["ids"], case["name"]
        assert ref.encode(case["text"], True) == case["ids_with_special"], case["name"]
        assert ref.decode(case["ids"], True) == case["decoded"], case["name"]


def test_corpus_covers_what_the_reference_says_it_covers():
    names = {c["name"] for c in CORPUS["cases"]}
    for n in ("empty", "french_accent", "rust_code", "emoji", "japanese", "arabic", "leading_spaces",
              "multiple_spaces", "newline_tab", "special_tokens", "image_token", "rare_unicode", "long_text",
              "repeated_char"):
        assert n in names
    assert CORPUS["generated_by"].startswith("tokenizers 0.23.3")


# ------------------------------------------------ unit cases (tokenizer.rs)
@pytest.mark.parametrize("text,expected", [
    ("hello", [23391]),
    ("Hello, world!", [9259, 236764, 1902, 236888]),
    ("Bonjour, le monde !", [53406, 236764, 674, 22150, 1717]),
    ("café", [123125, 236859]),
    ("😀 emoji", [242398, 64334]),
    ("  leading spaces", [138, 26016, 9952]),
    ("multiple   spaces", [43819, 139, 35220]),
    ("a\nb\tc", [236746, 107, 236763, 255968, 236755]),
    ("<bos>hello<eos>", [2, 23391, 1]),
    ("<|image|> a photo", [258880, 496, 4429]),
    ("\U0010FFFF", [482, 381, 429, 429]),
])
def test_encodes_reference_texts(mini, text, expected):
    assert mini.encode(text, False) == expected


def test_adds_bos_and_eos(mini):
    assert mini.encode("", True) == [2, 1]
    assert mini.encode("hello", True) == [2, 23391, 1]
    assert mini.encode("<bos>hello<eos>", True) == [2, 2, 23391, 1, 1]


def test_decodes_reference_texts(mini):
    assert mini.decode([23391], True) == "hello"
    assert mini.decode([2, 23391, 1], True) == "hello"
    assert mini.decode([2, 23391, 1], False) == "<bos>hello<eos>"
    assert mini.decode([258880, 496, 4429], True) == " a photo"


def test_exposes_special_ids(mini):
    assert (mini.bos_id(), mini.eos_id(), mini.unk_id(), mini.pad_id()) == (2, 1, 3, 0)
    assert mini.is_special_id(2) and not mini.is_special_id(23391)
    assert mini.token_id("<bos>") == 2 and mini.token(2) == "<bos>"
    assert mini.token_id("not a token") is None and mini.token(123456789) is None
    assert mini.vocab_size() == 694
    assert mini.max_token_id() == 258884


def test_byte_fallback_round_trips(mini):
    ids = mini.encode("\U0010FFFF", False)
    assert ids == [482, 381, 429, 429]
    assert mini.decode(ids, True) == "\U0010FFFF"


# ------------------------------------------------------------------ errors
@pytest.mark.parametrize("document", ["{}", '{"model":{"type":"Unigram"}}', "[]", "null"])
def test_rejects_documents_without_a_bpe_model(document):
    with pytest.raises((errors.CorruptError, errors.UnsupportedError)):
        Tokenizer.from_json_str(document)


@pytest.mark.parametrize("old,new,err", [
    ('"type":"BPE"', '"type":"Unigram"', errors.UnsupportedError),
    ('"byte_fallback":true', '"byte_fallback":false', errors.UnsupportedError),
    ('"fuse_unk":true', '"fuse_unk":false', errors.UnsupportedError),
    ('"ignore_merges":false', '"ignore_merges":true', errors.UnsupportedError),
    ('"dropout":null', '"dropout":0.1', errors.UnsupportedError),
    ('"behavior":"MergedWithPrevious"', '"behavior":"Isolated"', errors.UnsupportedError),
    ('"type":"TemplateProcessing"', '"type":"BertProcessing"', errors.UnsupportedError),
    ('"type":"ByteFallback"', '"type":"Strip"', errors.UnsupportedError),
    ('"<0x41>":', '"<0x41>x":', errors.CorruptError),        # a byte token missing
    ('"unk_token":"<unk>"', '"unk_token":"<nope>"', errors.CorruptError),
])
def test_rejects_unsupported_or_inconsistent_documents(old, new, err):
    """tokenizer.rs:1030-1056 and the loader's rules (tokenizer.rs:110-385):
    another pipeline is Unsupported, an inconsistent document Corrupt."""
    assert MINI.count(old) >= 1, old
    with pytest.raises(err):
        Tokenizer.from_json_str(MINI.replace(old, new, 1))


def test_rejects_inconsistent_merges_and_added_tokens():
    doc = json.loads(MINI)
    bad = json.loads(MINI)
    bad["model"]["merges"].append(["h", "zzz-not-a-token"])
    with pytest.raises(errors.CorruptError):
        Tokenizer.from_json_str(json.dumps(bad, ensure_ascii=False))
    bad = json.loads(MINI)
    bad["model"]["merges"].append(bad["model"]["merges"][0])
    with pytest.raises(errors.CorruptError, match="duplicate"):
        Tokenizer.from_json_str(json.dumps(bad, ensure_ascii=False))
    bad = json.loads(MINI)
    bad["added_tokens"].append(dict(bad["added_tokens"][0], content="<again>"))
    with pytest.raises(errors.CorruptError, match="duplicate added token id"):
        Tokenizer.from_json_str(json.dumps(bad, ensure_ascii=False))
    bad = json.loads(MINI)
    bad["added_tokens"][0]["id"] = 999999999
    with pytest.raises(errors.CorruptError, match="outside the vocabulary"):
        Tokenizer.from_json_str(json.dumps(bad, ensure_ascii=False))
    bad = json.loads(MINI)
    bad["model"]["vocab"]["<dup>"] = 2
    with pytest.raises(errors.CorruptError, match="duplicate tokenizer vocabulary id"):
        Tokenizer.from_json_str(json.dumps(bad, ensure_ascii=False))
    assert Tokenizer.from_json_str(json.dumps(doc, ensure_ascii=False)).vocab_size() == 694


@pytest.mark.parametrize("document", [
    '{"a":1,"a":2}', '{"a":[1,2,]}', '{"a":01}', '{"a":"\x01"}', '{"a":"\\ud800"}', '{"a":"\\udc00"}',
    '{"a":1} x', '{"a":NaN}', '{"a":1e999}', '{"a":tru}',
])
def test_the_json_reader_is_strict(document):
    """src/json/mod.rs: duplicate keys, trailing commas, leading zeros,
    control characters, lone surrogates, non-finite numbers and trailing
    content are Corrupt (before any tokenizer rule applies)."""
    with pytest.raises(errors.CorruptError, match="JSON"):
        Tokenizer.from_json_str(document)


def test_json_depth_cap():
    with pytest.raises(errors.LimitExceededError):
        Tokenizer.from_json_str("[" * 70 + "]" * 70)


def test_rejects_oversized_input(mini):
    with pytest.raises(errors.LimitExceededError):
        mini.encode("a" * (MAX_INPUT_BYTES + 1), False)


def test_rejects_too_many_tokens(mini):
    # 262,145 byte-fallback tokens from under 1 MiB of text
    with pytest.raises(errors.LimitExceededError, match="token cap"):
        mini.encode("\U0010FFFF" * 65537, False)


def test_rejects_unknown_ids_when_decoding(mini):
    with pytest.raises(errors.CorruptError):
        mini.decode([2**32 - 1], True)
    with pytest.raises(errors.CorruptError):
        mini.decode([-1], True)


def test_rejects_a_decoded_sequence_that_is_not_utf8(mini):
    # a lone continuation byte token
    with pytest.raises(errors.CorruptError, match="UTF-8"):
        mini.decode([mini.token_id("<0x80>")], True)


def test_the_c_abi_sizes_and_checks_its_buffers(mini):
    import ctypes

    lib = mini._lib
    n = ctypes.c_size_t()
    err = ctypes.create_string_buffer(256)
    ids = (ctypes.c_uint32 * 1)()
    rc = lib.svl_tokenizer_encode(mini._h, b"Hello, world!", 13, 0, ids, 1, ctypes.byref(n), err, 256)
    assert rc == errors.USAGE and n.value == 4
    rc = lib.svl_tokenizer_encode(mini._h, b"\xff", 1, 0, ids, 1, ctypes.byref(n), err, 256)
    assert rc == errors.USAGE and b"UTF-8" in err.value
    rc = lib.svl_tokenizer_create(b"\xff", 1, ctypes.byref(ctypes.c_void_p()), err, 256)
    assert rc == errors.CORRUPT
    out = ctypes.create_string_buffer(2)
    arr = (ctypes.c_uint32 * 1)(23391)
    rc = lib.svl_tokenizer_decode(mini._h, arr, 1, 1, out, 2, ctypes.byref(n), err, 256)
    assert rc == errors.USAGE and n.value == 5


# ----------------------------------------- merge loop vs. the reference loop
def _alphabet(ref):
    chars = sorted({c for case in CORPUS["cases"] for c in case["text"]})
    return chars + ["▁", "ÿ", "一", "\U0001F600", "<bos>", "<|image|>"]


@pytest.mark.parametrize("seed", range(6))
def test_heap_merges_equal_the_reference_loop_on_random_text(mini, ref, seed):
    """The product's O(n log n) merge loop against the reference's quadratic
    rounds on seeded random strings over the corpus alphabet, long runs of
    one character (overlapping pairs) and added-token markers included."""
    rnd = random.Random(seed)
    alpha = _alphabet(ref)
    for _ in range(40):
        n = rnd.randint(0, 300)
        if rnd.random() < 0.3:
            text = rnd.choice(alpha) * n
        else:
            text = "".join(rnd.choice(alpha) for _ in range(n))
        for special in (False, True):
            got = mini.encode(text, special)
            assert got == ref.encode(text, special), text
        assert mini.decode(got, True) == ref.decode(got, True)


def test_heap_merges_equal_the_reference_loop_on_corpus_mixtures(mini, ref):
    rnd = random.Random(7)
    texts = [c["text"] for c in CORPUS["cases"]]
    for _ in range(60):
        text = " ".join(rnd.choice(texts)[: rnd.randint(0, 400)] for _ in range(rnd.randint(1, 4)))
        assert mini.encode(text, True) == ref.encode(text, True)


# ------------------------------------------------------ prompts (prompt.rs)
def test_prefixes_match_the_official_configuration():
    assert prompt.SEARCH_QUERY == "task: search result | query: "
    assert prompt.DOCUMENT == "title: none | text: "
    assert prompt.CLASSIFICATION == "task: classification | query: "
    assert prompt.CLUSTERING == "task: clustering | query: "
    assert prompt.CODE_RETRIEVAL == "task: code retrieval | query: "
    assert prompt.FACT_CHECKING == "task: fact checking | query: "
    assert prompt.SENTENCE_SIMILARITY == "task: sentence similarity | query: "
    assert prompt.QUESTION_ANSWERING == "task: question answering | query: "


def test_prompt_roles_and_names():
    assert prompt.Prompt.SearchQuery.prefix() == prompt.SEARCH_QUERY
    assert prompt.Prompt.SearchQuery.is_query() and not prompt.Prompt.Document.is_query()
    assert prompt.Prompt.from_name("CodeRetrieval") is prompt.Prompt.CodeRetrieval
    assert prompt.Prompt.from_name("searchquery") is None and prompt.Prompt.from_name("unknown") is None
    assert prompt.apply(prompt.Prompt.SearchQuery, "hello") == "task: search result | query: hello"
    assert prompt.apply(prompt.Prompt.Document, "hello") == "title: none | text: hello"


def test_token_id_golden_cases_carry_the_official_prefixes():
    """The real-model golden cases (fixtures/model/text_golden.json) were
    tokenised from prefix + text with <bos> / <eos>."""
    cases = json.loads((GOLDEN / "token_ids.json").read_text(encoding="utf-8"))["cases"]
    for c in cases:
        assert prompt.Prompt.from_name(c["prompt"]).prefix() == c["prefix"]
        assert c["token_ids"][0] == 2 and c["token_ids"][-1] == 1


def test_damaged_documents_never_crash_the_loader():
    """Random byte changes and truncations of the tokenizer document load, or
    fail with one of the reference's error variants (a truncated or mangled
    JSON is Corrupt; a changed pipeline Unsupported; invalid UTF-8 Corrupt)."""
    rnd = random.Random(5)
    data = MINI.encode("utf-8")
    ok = 0
    for trial in range(400):
        d = bytearray(data)
        if trial % 2:
            del d[rnd.randrange(len(d)):]
        else:
            for _ in range(rnd.randint(1, 3)):
                d[rnd.randrange(len(d))] = rnd.randrange(32, 127)
        try:
            t = Tokenizer.from_json_bytes(bytes(d))
        except (errors.CorruptError, errors.UnsupportedError, errors.LimitExceededError):
            continue
        ok += 1
        t.encode("Hello, world! café 😀", True)
    assert ok < 400


@pytest.mark.parametrize("seed", range(3))
def test_random_text_never_crashes_encode_and_round_trips(mini, seed):
    """Arbitrary scalar values (byte fallback for anything outside the reduced
    vocabulary) encode, and decoding gives the text back."""
    rnd = random.Random(100 + seed)
    for _ in range(100):
        chars = []
        for _ in range(rnd.randint(0, 80)):
            cp = rnd.choice([rnd.randint(0x20, 0x7E), rnd.randint(0xA0, 0xD7FF), rnd.randint(0xE000, 0x10FFFF)])
            chars.append(chr(cp))
        text = "".join(chars)
        ids = mini.encode(text, True)
        assert mini.decode(ids, True) == text


@pytest.mark.parametrize("threads", [1, 3, 0])
def test_batch_encode_equals_per_text_encode(mini, threads):
    """svl_tokenizer_encode_batch: the packed ids of per-text encode calls,
    whatever the number of host threads."""
    rnd = random.Random(threads)
    texts = [c["text"] for c in CORPUS["cases"]] * 3
    texts += ["".join(chr(rnd.randint(0x20, 0x2FF)) for _ in range(rnd.randint(0, 50))) for _ in range(40)]
    rnd.shuffle(texts)
    for special in (False, True):
        ids, cu = mini.encode_batch(texts, special, threads)
        assert cu.size == len(texts) + 1 and cu[0] == 0 and int(cu[-1]) == ids.size
        for i, t in enumerate(texts):
            assert ids[cu[i]:cu[i + 1]].tolist() == mini.encode(t, special)
    ids, cu = mini.encode_batch([], True, threads)
    assert ids.size == 0 and cu.tolist() == [0]


def test_batch_encode_reports_the_first_failing_text(mini):
    texts = ["hello", "a" * (MAX_INPUT_BYTES + 1), "b" * (MAX_INPUT_BYTES + 1), "world"]
    with pytest.raises(errors.LimitExceededError, match="text 1"):
        mini.encode_batch(texts, True, 4)


def test_embedder_tokenises_many_texts_as_one_at_a_time(mini):
    """TextEmbedder.embed_many / ingest tokenise with one batched call; the
    packed ids are those of per-text token_ids (prefix, <bos>, <eos>)."""
    from svl.prompt import Prompt
    from svl.text import TextEmbedder

    emb = TextEmbedder(None, mini)
    texts = [c["text"] for c in CORPUS["cases"]]
    for p in (Prompt.Document, Prompt.SearchQuery):
        ids, cu = emb.token_ids_many(texts, p)
        for i, t in enumerate(texts):
            assert ids[cu[i]:cu[i + 1]].tolist() == emb.token_ids(t, p).tolist()
