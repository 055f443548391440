"""Writes ``production_embeddings.json``: CPU-oracle embeddings of the
24-layer production-shaped encoder at the benchmark's own sequence lengths.

The model is the benchmark's: the frozen manifest's shapes with random
N(0, 0.02) weights drawn from ``default_rng(1234)`` (``svl.synth``).  The
sequences are

* four sequences of the BASELINE configs[1] batch (``svl.synth.config2_batch``,
  seed 2): index 12 (509 tokens, the longest), 0 (440), 3 (198) and the
  shortest one; the GPU tests embed the whole 64-sequence batch, as the
  benchmark does, and compare these four;
* the first 2048-token sequence of BASELINE configs[2]
  (``svl.synth.config3_batch``, seed 3), where the 512-token sliding window
  masks whole key blocks.

Each embedding is the oracle's ``embed_ids(ids, 768)``: ``normalized``
truncated and renormalised at 768 (``ForwardOutput::embedding``,
text.rs:72-74), 768 floats of the reference's scalar FP32 path restated in
``oracle/``.  Generating them takes
about two minutes of CPU on 8 threads, which is why they are committed rather
than recomputed in every GPU run; ``tests/test_oracle_golden.py`` re-derives
the shortest one to pin the file to the oracle.

Usage: ``python tests/golden/make_production_golden.py``
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (str(ROOT), str(ROOT / "seldon-vault-lite-rust_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

OUT = HERE / "production_embeddings.json"


def cases():
    """(name, source, index, ids) of every fixture sequence."""
    from svl import synth

    batch = synth.config2_batch()
    lengths = [len(s) for s in batch]
    shortest = int(np.argmin(lengths))
    out = [(f"configs1[{i}]", "configs1", i, batch[i]) for i in (12, 0, 3, shortest)]
    out.append(("configs2[0]", "configs2", 0, synth.config3_batch()[0]))
    return out


def main() -> None:
    import oracle
    from svl import synth
    from svl.text import pack

    cfg = synth.manifest_config()
    w = synth.random_weights(cfg, seed=1234)
    orc = oracle.OracleModel(cfg, w)
    cs = cases()
    ids, cu = pack([c[3] for c in cs])
    emb = orc.embed_many(ids, cu, cfg.embedding_dim, threads=len(cs))
    doc = {
        "model": "manifest shapes, random N(0, 0.02) weights, default_rng(1234)",
        "cases": [
            {"name": c[0], "source": c[1], "index": c[2], "length": int(len(c[3])),
             "embedding": [float(x) for x in emb[i]]}
            for i, c in enumerate(cs)
        ],
    }
    OUT.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {OUT} ({len(cs)} cases)")


if __name__ == "__main__":
    main()
