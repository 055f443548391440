"""Pure-Python restatement of the reference tokenizer's encode and decode.

TEST INFRASTRUCTURE ONLY.  Imported by tests/ as the checker of the C++
tokenizer in libsvl_gpu.so (seldon-vault-lite-rust_b200/csrc/tokenizer.cpp),
never by the product.  It follows src/model/tokenizer.rs step by step,
including its quadratic merge loop (tokenizer.rs:520-560: find the adjacent
pair of lowest merge rank, merge all of its non-overlapping occurrences left
to right, repeat), which the product replaces with an equivalent heap; the
random-text tests compare the two.  Loader validation is not restated (the
product's own tests cover it against the reference's rules).

Parity pin: tests/test_tokenizer.py checks this restatement against the
reference's golden corpus (tests/golden/tokenizer/golden.json, produced by
the official tokenizers library) before using it on other text.
"""

from __future__ import annotations

import json

MARKER = "▁"


class RefTokenizer:
    def __init__(self, document: str):
        root = json.loads(document)
        model = root["model"]
        self.vocab = {tok: int(i) for tok, i in model["vocab"].items()}
        self.id_to_token = {i: tok for tok, i in self.vocab.items()}
        # one-character tokens (tokenizer.rs:204-212)
        self.char_ids = {tok: i for tok, i in self.vocab.items() if len(tok) == 1}
        self.byte_ids = [self.vocab[f"<0x{b:02X}>"] for b in range(256)]
        # (left id, right id) -> (rank, merged id)  (tokenizer.rs:236-270)
        self.merges = {}
        for rank, (left, right) in enumerate(model["merges"]):
            self.merges[(self.vocab[left], self.vocab[right])] = (rank, self.vocab[left + right])
        # added tokens, longest first then by id (tokenizer.rs:345-351)
        self.added = sorted(((t["content"], int(t["id"])) for t in root["added_tokens"]),
                            key=lambda a: (-len(a[0].encode("utf-8")), a[1]))
        self.special = {int(t["id"]) for t in root["added_tokens"] if t["special"]}
        self.bos = self.vocab["<bos>"]
        self.eos = self.vocab["<eos>"]

    # tokenizer.rs:392-434
    def encode(self, text: str, add_special: bool) -> list[int]:
        ids = [self.bos] if add_special else []
        segment = []
        data = text.encode("utf-8")
        i = 0
        while i < len(data):
            hit = next(((t, tid) for t, tid in self.added if data.startswith(t.encode("utf-8"), i)), None)
            if hit is not None:
                if segment:
                    ids += self._segment("".join(segment))
                    segment = []
                ids.append(hit[1])
                i += len(hit[0].encode("utf-8"))
                continue
            # one character (its UTF-8 length from the lead byte)
            b = data[i]
            n = 1 if b < 0x80 else 2 if b < 0xE0 else 3 if b < 0xF0 else 4
            segment.append(data[i:i + n].decode("utf-8"))
            i += n
        if segment:
            ids += self._segment("".join(segment))
        if add_special:
            ids.append(self.eos)
        return ids

    # tokenizer.rs:520-560
    def _segment(self, segment: str) -> list[int]:
        symbols = []
        for ch in segment:
            norm = MARKER if ch == " " else ch
            if norm in self.char_ids:
                symbols.append(self.char_ids[norm])
            else:
                symbols += [self.byte_ids[b] for b in norm.encode("utf-8")]
        while True:
            best = None
            for a, b in zip(symbols, symbols[1:]):
                m = self.merges.get((a, b))
                if m is not None and (best is None or m[0] < best[0]):
                    best = (m[0], a, b, m[1])
            if best is None:
                return symbols
            _, left, right, merged = best
            out, k = [], 0
            while k < len(symbols):
                if k + 1 < len(symbols) and symbols[k] == left and symbols[k + 1] == right:
                    out.append(merged)
                    k += 2
                else:
                    out.append(symbols[k])
                    k += 1
            symbols = out

    # tokenizer.rs:441-466
    def decode(self, ids, skip_special: bool) -> str:
        out = bytearray()
        for i in ids:
            tok = self.id_to_token[i]
            if skip_special and i in self.special:
                continue
            if len(tok) == 6 and tok.startswith("<0x") and tok.endswith(">"):
                out.append(int(tok[3:5], 16))
                continue
            out += tok.replace(MARKER, " ").encode("utf-8")
        return out.decode("utf-8")
