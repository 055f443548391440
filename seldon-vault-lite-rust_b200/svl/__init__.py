"""svl -- B200 (sm_100a) text-embedding and exact-search hot path of Seldon
Vault Lite, behind the reference crate's embed / vector-search API.

Host-side mirror of the reference interfaces over the C ABI of
libsvl_gpu.so (include/svl_gpu.h):

* svl.text.TextModel / ForwardOutput   -- src/model/text.rs
* svl.text.TextEmbedder                -- text.rs:590-626 (prompt + tokenizer + model)
* svl.tokenizer.Tokenizer              -- src/model/tokenizer.rs (include/svl_tokenizer.h)
* svl.prompt.Prompt / apply            -- src/model/prompt.rs
* svl.bundle.Bundle / load_text_model  -- src/bundle/mod.rs, src/model/source.rs (include/svl_bundle.h)
* svl.index.VectorIndex / rank / Index -- src/index/vector.rs, src/index/mod.rs
* svl.config.TextConfig                -- src/model/config.rs
* svl.errors                           -- src/error.rs
* svl.dist                             -- data-parallel encoder and row-sharded
                                          search over one process per GPU
"""

from . import errors
from .config import TextConfig

__all__ = ["errors", "TextConfig"]
