"""Strict parser of the EmbeddingGemma-2 text configuration.

Mirrors ``TextConfig::from_json_value`` (reference src/model/config.rs:112-269):
the same required keys, the same caps, the same per-layer overrides, the
"last layer must be full" rule (config.rs:648) and the same derived f32
constants (embedding_scale = sqrt(hidden_size), ple_scale = 1 / that,
config.rs:241-242).  Violations raise the same error variants.
"""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import errors

MAX_CONFIG_BYTES = 1024 * 1024
MAX_TEXT_TOKENS = 8192  # config.rs:27
MAX_HIDDEN_SIZE = 16384
MAX_LAYERS = 128
MAX_HEADS = 128
MAX_HEAD_DIM = 1024
MAX_INTERMEDIATE_SIZE = 65536
MAX_VOCAB_SIZE = 1_000_000
MAX_EMBEDDING_DIM = 16384
MAX_POSITIONS = 1_048_576

SLIDING = 0
FULL = 1


@dataclass(frozen=True)
class LayerConfig:
    layer_type: int  # SLIDING or FULL
    head_dim: int
    num_key_value_heads: int


@dataclass
class TextConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    hidden_size_per_layer_input: int
    embedding_dim: int
    max_position_embeddings: int
    rms_norm_eps: float
    sliding_window: int
    pad_token_id: int | None
    bos_token_id: int | None
    eos_token_id: int | None
    full_rope_theta: float
    sliding_rope_theta: float
    layers: list[LayerConfig] = field(default_factory=list)

    # f32 constants exactly as config.rs:241-242 computes them
    @property
    def embedding_scale(self) -> float:
        return float(np.sqrt(np.float32(self.hidden_size)))

    @property
    def ple_scale(self) -> float:
        return float(np.float32(1.0) / np.float32(self.embedding_scale))

    # ------------------------------------------------------------------ parse
    @classmethod
    def from_json_str(cls, text: str) -> "TextConfig":
        if len(text.encode()) > MAX_CONFIG_BYTES:
            raise errors.LimitExceededError("configuration file above the 1 MiB cap")
        try:
            value = json.loads(text)
        except json.JSONDecodeError as exc:
            raise errors.CorruptError(f"configuration is not valid JSON: {exc}") from None
        return cls.from_json_value(value)

    @classmethod
    def from_file(cls, path: str | Path) -> "TextConfig":
        return cls.from_json_str(Path(path).read_text())

    @classmethod
    def from_json_value(cls, value) -> "TextConfig":
        if not isinstance(value, dict):
            raise errors.CorruptError("model configuration must be a JSON object")
        text = value.get("text_config", value)
        if not isinstance(text, dict):
            raise errors.CorruptError("text_config must be a JSON object")
        if "model_type" in text and text["model_type"] != "embedding_gemma2_text":
            raise errors.UnsupportedError(f"text model type {text['model_type']} is not embedding_gemma2_text")
        if "dtype" in text:
            dtype = text["dtype"]
            if dtype == "float16":
                raise errors.UnsupportedError("float16 is forbidden for EmbeddingGemma 2 activations")
            if dtype not in ("bfloat16", "float32"):
                raise errors.UnsupportedError(f"model dtype {dtype} is not supported")

        hidden = _unsigned(text, "hidden_size")
        inter = _unsigned(text, "intermediate_size")
        n_layers = _unsigned(text, "num_hidden_layers")
        n_heads = _unsigned(text, "num_attention_heads")
        g_kv = _unsigned(text, "num_key_value_heads")
        g_hd = _unsigned(text, "head_dim")
        ple = _unsigned(text, "hidden_size_per_layer_input")
        emb = _unsigned(text, "embedding_dim")
        vocab = _unsigned(text, "vocab_size")
        max_pos = _unsigned(text, "max_position_embeddings")
        window = _unsigned(text, "sliding_window")
        eps = _float(text, "rms_norm_eps")
        if not np.isfinite(np.float32(eps)):
            raise errors.CorruptError("RMSNorm epsilon does not fit a finite f32 value")
        if _string(text, "hidden_activation") != "gelu_pytorch_tanh":
            raise errors.UnsupportedError("hidden activation is not gelu_pytorch_tanh")
        if text.get("attention_bias", False) is True:
            raise errors.UnsupportedError("attention bias is not part of the frozen model")
        if "attention_dropout" in text and float(text["attention_dropout"]) != 0.0:
            raise errors.UnsupportedError("attention dropout is not implemented by the inference engine")

        _cap(hidden, MAX_HIDDEN_SIZE, "hidden size")
        _cap(inter, MAX_INTERMEDIATE_SIZE, "intermediate size")
        _cap(n_layers, MAX_LAYERS, "layer count")
        _cap(n_heads, MAX_HEADS, "attention head count")
        _cap(ple, MAX_HIDDEN_SIZE, "per-layer input size")
        _cap(emb, MAX_EMBEDDING_DIM, "embedding dimension")
        _cap(vocab, MAX_VOCAB_SIZE, "vocabulary size")
        _cap(max_pos, MAX_POSITIONS, "position count")
        if window == 0 or window > max_pos:
            raise errors.LimitExceededError(f"sliding window {window} is outside 1..={max_pos}")
        if not np.isfinite(eps) or eps < 0:
            raise errors.CorruptError("RMSNorm epsilon must be finite and non-negative")
        _validate_head_layout(n_heads, g_kv, g_hd)

        types = text.get("layer_types")
        if types is None:
            raise errors.CorruptError("layer_types is missing")
        if not isinstance(types, list):
            raise errors.CorruptError("layer_types must be an array")
        if len(types) != n_layers:
            raise errors.CorruptError(f"layer_types has {len(types)} entries, expected {n_layers}")
        parsed_types = []
        for name in types:
            if name == "sliding_attention":
                parsed_types.append(SLIDING)
            elif name == "full_attention":
                parsed_types.append(FULL)
            else:
                raise errors.UnsupportedError(f"layer type {name} is not sliding_attention or full_attention")
        if parsed_types[-1] != FULL:
            raise errors.UnsupportedError("the last layer must use full attention")

        overrides = {}
        plc = text.get("per_layer_config")
        if plc is not None:
            if not isinstance(plc, dict):
                raise errors.CorruptError("per_layer_config must be an object")
            for key, entry in plc.items():
                try:
                    index = int(key)
                except ValueError:
                    raise errors.CorruptError(f"per_layer_config key {key} is not an index") from None
                if index < 0 or index >= n_layers:
                    raise errors.CorruptError(f"per_layer_config index {index} is outside {n_layers} layers")
                overrides[index] = (_unsigned(entry, "head_dim"), _unsigned(entry, "num_key_value_heads"))
        layers = []
        for i, lt in enumerate(parsed_types):
            hd, kv = overrides.get(i, (g_hd, g_kv))
            _validate_head_layout(n_heads, kv, hd)
            layers.append(LayerConfig(lt, hd, kv))
        for lt in (SLIDING, FULL):  # config.rs validate_uniform_head_dim
            dims = {l.head_dim for l in layers if l.layer_type == lt}
            if len(dims) > 1:
                raise errors.UnsupportedError("layers of the same attention type must share one head dimension")

        rope = text.get("rope_parameters")
        if rope is None:
            raise errors.CorruptError("rope_parameters is missing")
        full_theta = sliding_theta = None
        for key, entry in rope.items():
            if _string(entry, "rope_type") != "default":
                raise errors.UnsupportedError("RoPE type is not supported")
            theta = _float(entry, "rope_theta")
            if not np.isfinite(theta) or theta <= 1.0:
                raise errors.CorruptError(f"RoPE theta {theta} must be finite and greater than one")
            if key == "full_attention":
                full_theta = theta
            elif key == "sliding_attention":
                sliding_theta = theta
            else:
                raise errors.UnsupportedError(f"RoPE parameters for {key} are not supported")
        if full_theta is None or sliding_theta is None:
            raise errors.CorruptError("rope_parameters must declare full_attention and sliding_attention")

        specials = [_optional_token(text, k) for k in ("pad_token_id", "bos_token_id", "eos_token_id")]
        for sid in specials:
            if sid is not None and sid >= vocab:
                raise errors.CorruptError(f"special token id {sid} is outside the vocabulary of {vocab} entries")
        return cls(
            vocab_size=vocab,
            hidden_size=hidden,
            intermediate_size=inter,
            num_hidden_layers=n_layers,
            num_attention_heads=n_heads,
            hidden_size_per_layer_input=ple,
            embedding_dim=emb,
            max_position_embeddings=max_pos,
            rms_norm_eps=float(np.float32(eps)),
            sliding_window=window,
            pad_token_id=specials[0],
            bos_token_id=specials[1],
            eos_token_id=specials[2],
            full_rope_theta=float(np.float32(full_theta)),
            sliding_rope_theta=float(np.float32(sliding_theta)),
            layers=layers,
        )

    # ------------------------------------------------------------ inventory
    def tensor_shapes(self) -> list[tuple[str, tuple[int, ...]]]:
        """Expected text tensors and shapes (config.rs:394-484)."""
        h, p, f = self.hidden_size, self.hidden_size_per_layer_input, self.intermediate_size
        out = [
            ("language_model.embed_tokens.weight", (self.vocab_size, h)),
            ("language_model.embedding_projection.weight", (self.embedding_dim, h)),
            ("language_model.norm.weight", (h,)),
            ("language_model.ple.per_layer_model_projection.weight", (self.num_hidden_layers * p, h)),
            ("language_model.ple.per_layer_projection_norm.weight", (p,)),
        ]
        for i, layer in enumerate(self.layers):
            pre = f"language_model.layers.{i}"
            q = self.num_attention_heads * layer.head_dim
            kv = layer.num_key_value_heads * layer.head_dim
            out += [
                (f"{pre}.input_layernorm.weight", (h,)),
                (f"{pre}.post_attention_layernorm.weight", (h,)),
                (f"{pre}.pre_feedforward_layernorm.weight", (h,)),
                (f"{pre}.post_feedforward_layernorm.weight", (h,)),
                (f"{pre}.layer_scalar", (1,)),
                (f"{pre}.mlp.gate_proj.weight", (f, h)),
                (f"{pre}.mlp.up_proj.weight", (f, h)),
                (f"{pre}.mlp.down_proj.weight", (h, f)),
                (f"{pre}.ple_block.per_layer_input_gate.weight", (p, h)),
                (f"{pre}.ple_block.per_layer_projection.weight", (h, p)),
                (f"{pre}.ple_block.post_per_layer_input_norm.weight", (h,)),
                (f"{pre}.self_attn.q_proj.weight", (q, h)),
                (f"{pre}.self_attn.k_proj.weight", (kv, h)),
                (f"{pre}.self_attn.v_proj.weight", (kv, h)),
                (f"{pre}.self_attn.o_proj.weight", (h, q)),
                (f"{pre}.self_attn.q_norm.weight", (layer.head_dim,)),
                (f"{pre}.self_attn.k_norm.weight", (layer.head_dim,)),
            ]
        return out

    # ------------------------------------------------------------------ ABI
    def to_c(self):
        """Returns (svl_text_config, keepalive) for the C ABI."""
        from ._abi import SvlLayerConfig, SvlTextConfig

        layer_arr = (SvlLayerConfig * self.num_hidden_layers)(
            *[SvlLayerConfig(l.layer_type, l.head_dim, l.num_key_value_heads) for l in self.layers]
        )
        c = SvlTextConfig(
            vocab_size=self.vocab_size,
            hidden_size=self.hidden_size,
            intermediate_size=self.intermediate_size,
            num_hidden_layers=self.num_hidden_layers,
            num_attention_heads=self.num_attention_heads,
            hidden_size_per_layer_input=self.hidden_size_per_layer_input,
            embedding_dim=self.embedding_dim,
            max_position_embeddings=self.max_position_embeddings,
            sliding_window=self.sliding_window,
            pad_token_id=-1 if self.pad_token_id is None else self.pad_token_id,
            rms_norm_eps=self.rms_norm_eps,
            embedding_scale=self.embedding_scale,
            ple_scale=self.ple_scale,
            full_rope_theta=self.full_rope_theta,
            sliding_rope_theta=self.sliding_rope_theta,
            layers=ctypes.cast(layer_arr, ctypes.POINTER(SvlLayerConfig)),
        )
        return c, layer_arr

    def linear_flops_per_token(self) -> int:
        """2 x the MACs of every projection one token goes through (PLE, q/k/v,
        o, gate/up, down, the two PLE-block projections, the final 512->768)."""
        h, p, f, e = self.hidden_size, self.hidden_size_per_layer_input, self.intermediate_size, self.embedding_dim
        macs = h * self.num_hidden_layers * p + h * e
        for layer in self.layers:
            q, kv = self.num_attention_heads * layer.head_dim, layer.num_key_value_heads * layer.head_dim
            macs += h * (q + 2 * kv) + q * h + 2 * h * f + f * h + 2 * h * p
        return 2 * macs

    def linear_flops_split_per_token(self, fp16: bool = True) -> tuple:
        """(FP16-operand, TF32-operand) parts of linear_flops_per_token.  With
        the library's default operand placement every projection runs on FP16
        operands with power-of-two row scales; SVL_GEMM_TF32=1 (fp16=False)
        puts them all on TF32 operands."""
        total = self.linear_flops_per_token()
        return (total, 0) if fp16 else (0, total)

    def attention_flops(self, length: int) -> int:
        return self.flops_per_sequence(length) - length * self.linear_flops_per_token()

    def flops_per_sequence(self, length: int) -> int:
        """Algorithmic FLOPs of one forward at `length` tokens: 2 x MACs of
        every linear plus 2 x (QK^T + PV) MACs over the attended window."""
        h, p, f, e = self.hidden_size, self.hidden_size_per_layer_input, self.intermediate_size, self.embedding_dim
        n = self.num_attention_heads
        macs = length * (h * self.num_hidden_layers * p + h * e)
        for layer in self.layers:
            q, kv = n * layer.head_dim, layer.num_key_value_heads * layer.head_dim
            macs += length * (h * (q + 2 * kv) + q * h + 2 * h * f + f * h + 2 * h * p)
            if layer.layer_type == FULL:
                attended = length * length
            else:
                w = self.sliding_window
                i = np.arange(length, dtype=np.int64)
                attended = int((np.minimum(length - 1, i + w) - np.maximum(0, i - w) + 1).sum())
            macs += 2 * n * layer.head_dim * attended
        return 2 * int(macs)


def _unsigned(obj, key):
    if key not in obj:
        raise errors.CorruptError(f"configuration is missing {key}")
    v = obj[key]
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        if isinstance(v, float) and v.is_integer() and v >= 0:
            return int(v)
        raise errors.CorruptError(f"{key} must be a non-negative integer")
    return v


def _float(obj, key):
    if key not in obj:
        raise errors.CorruptError(f"configuration is missing {key}")
    v = obj[key]
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        raise errors.CorruptError(f"{key} must be a number")
    return float(v)


def _string(obj, key):
    if key not in obj:
        raise errors.CorruptError(f"configuration is missing {key}")
    v = obj[key]
    if not isinstance(v, str):
        raise errors.CorruptError(f"{key} must be a string")
    return v


def _optional_token(obj, key):
    v = obj.get(key)
    if v is None:
        return None
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise errors.CorruptError(f"{key} must be a non-negative integer")
    if v > 0xFFFFFFFF:
        raise errors.LimitExceededError(f"{key} does not fit u32")
    return v


def _cap(value, cap, label):
    if value == 0 or value > cap:
        raise errors.LimitExceededError(f"{label} {value} is outside 1..={cap}")


def _validate_head_layout(n_heads, kv, hd):
    if kv == 0 or kv > n_heads:
        raise errors.CorruptError(f"key/value head count {kv} is not in 1..={n_heads}")
    if n_heads % kv:
        raise errors.CorruptError("attention head count is not a multiple of key/value head count")
    if hd == 0 or hd > MAX_HEAD_DIM or hd % 2:
        raise errors.CorruptError(f"head dimension {hd} must be a positive even value at most {MAX_HEAD_DIM}")
