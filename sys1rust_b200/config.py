"""Model configuration: the ModernBERT encoder config plus the decision-head shape.

Mirrors ``EncoderConfig`` / ``AgentConfig`` of the reference runtime
(``runtime/crates/laya-core/src/config.rs:9-202``): the same field names, the same
defaults, the same normalisation of the transformers 4.x (``global_rope_theta``) and 5.x
(``rope_parameters``) layouts, the same layer pattern rule (``layer_types`` first, else
``i % global_attn_every_n_layers != 0`` is local, ``config.rs:135-141``) and the same
shape checks with the same error texts (``config.rs:165-192``).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


class ConfigError(ValueError):
    """A checkpoint config that the backend cannot run (``Error::Config`` in the reference)."""


@dataclass
class EncoderConfig:
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    intermediate_size: int
    norm_eps: float = 1e-5
    global_attn_every_n_layers: int = 3
    # Sliding window width in tokens: a query attends keys within local_attention // 2.
    local_attention: int = 128
    global_rope_theta: float = 160000.0
    local_rope_theta: float = 10000.0
    pad_token_id: int = 0
    max_position_embeddings: int = 8192
    layer_is_local: List[bool] = field(default_factory=list)

    @staticmethod
    def from_value(v: Dict[str, Any]) -> "EncoderConfig":
        """Parse ``encoder/config.json`` (``config.rs:95-163``)."""
        def get_u(k: str) -> int:
            x = v.get(k)
            if not isinstance(x, int) or isinstance(x, bool) or x < 0:
                raise ConfigError(f"encoder config: missing integer '{k}'")
            return x

        def get_f(k: str, d: float) -> float:
            x = v.get(k)
            return float(x) if isinstance(x, (int, float)) and not isinstance(x, bool) else d

        if v.get("model_type") != "modernbert":
            raise ConfigError(
                f"unsupported encoder model_type {v.get('model_type')!r}; only 'modernbert' is implemented")
        n_layers = get_u("num_hidden_layers")
        every = v.get("global_attn_every_n_layers", 3)
        if not isinstance(every, int):
            every = 3
        if every == 0:
            raise ConfigError("encoder config: global_attn_every_n_layers must be at least 1")
        g_theta = get_f("global_rope_theta", 160000.0)
        l_theta = get_f("local_rope_theta", 10000.0)
        rp = v.get("rope_parameters")
        if isinstance(rp, dict):
            t = (rp.get("full_attention") or {}).get("rope_theta")
            if isinstance(t, (int, float)):
                g_theta = float(t)
            t = (rp.get("sliding_attention") or {}).get("rope_theta")
            if isinstance(t, (int, float)):
                l_theta = float(t)
        types = v.get("layer_types")
        if isinstance(types, list) and len(types) == n_layers:
            local = [t == "sliding_attention" for t in types]
        else:
            local = [i % every != 0 for i in range(n_layers)]
        la = v.get("local_attention", 128)
        mpe = v.get("max_position_embeddings", 8192)
        cfg = EncoderConfig(
            vocab_size=get_u("vocab_size"),
            hidden_size=get_u("hidden_size"),
            num_hidden_layers=n_layers,
            num_attention_heads=get_u("num_attention_heads"),
            intermediate_size=get_u("intermediate_size"),
            norm_eps=get_f("norm_eps", get_f("layer_norm_eps", 1e-5)),
            global_attn_every_n_layers=every,
            local_attention=la if isinstance(la, int) else 128,
            global_rope_theta=g_theta,
            local_rope_theta=l_theta,
            pad_token_id=int(v.get("pad_token_id") or 0),
            max_position_embeddings=mpe if isinstance(mpe, int) else 8192,
            layer_is_local=local,
        )
        cfg.check_shapes()
        return cfg

    def check_shapes(self) -> None:
        """The divisibility rules of ``config.rs:165-192``, same messages."""
        def bad(msg: str) -> None:
            raise ConfigError(f"encoder config: {msg}")

        if self.num_attention_heads == 0:
            bad("num_attention_heads must be at least 1")
        if self.hidden_size == 0:
            bad("hidden_size must be at least 1")
        if self.hidden_size % self.num_attention_heads != 0:
            bad(f"hidden_size {self.hidden_size} is not a multiple of num_attention_heads "
                f"{self.num_attention_heads}")
        if self.hidden_size % self.head_nheads() != 0:
            bad(f"hidden_size {self.hidden_size} is not a multiple of the {self.head_nheads()} "
                f"decision-head attention heads (max(1, hidden_size // 64))")
        if self.local_attention < 2:
            bad("local_attention must be at least 2")

    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def head_nheads(self) -> int:
        """Decision-head attention heads, ``max(1, d // 64)`` (``config.rs:199-201``)."""
        return max(1, self.hidden_size // 64)

    def window(self) -> int:
        """Half-width of the sliding window: |i - j| <= window (``lib.rs:1122``)."""
        return self.local_attention // 2

    def to_value(self) -> Dict[str, Any]:
        return {
            "model_type": "modernbert",
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "intermediate_size": self.intermediate_size,
            "norm_eps": self.norm_eps,
            "global_attn_every_n_layers": self.global_attn_every_n_layers,
            "local_attention": self.local_attention,
            "global_rope_theta": self.global_rope_theta,
            "local_rope_theta": self.local_rope_theta,
            "pad_token_id": self.pad_token_id,
            "max_position_embeddings": self.max_position_embeddings,
            "layer_types": ["sliding_attention" if l else "full_attention" for l in self.layer_is_local],
        }


@dataclass
class ModelConfig:
    """Encoder config plus the decision-head facts a backend needs (``config.rs:205-209``)."""
    encoder: EncoderConfig
    head_layers: int = 2
    max_len: int = 512
    head_max_len: int = 192
    # Width of the head FFN (``head.layers.{j}.linear1.weight`` rows) and of the scorer's
    # hidden layer (``scorer.1.weight`` rows); both are read from the weights in the reference.
    head_ffn: int = 4096
    scorer_hidden: int = 256
    n_qtypes: int = 3

    @staticmethod
    def load(model_dir: str) -> "ModelConfig":
        p = os.path.join(model_dir, "rl_agent_config.json")
        if not os.path.exists(p):
            raise ConfigError(
                f"Incompatible model: {model_dir} does not contain 'rl_agent_config.json'. "
                "That file ships with the weights of a Laya checkpoint.")
        with open(p) as f:
            agent = json.load(f)
        ep = os.path.join(model_dir, "encoder", "config.json")
        if not os.path.exists(ep):
            raise ConfigError(f"missing encoder config {ep}")
        with open(ep) as f:
            enc = EncoderConfig.from_value(json.load(f))
        return ModelConfig(encoder=enc,
                           head_layers=int(agent.get("head_layers", 2)),
                           max_len=int(agent.get("max_len", 512)),
                           head_max_len=int(agent.get("head_max_len", 192)),
                           head_ffn=int(agent.get("head_ffn", 4 * enc.hidden_size)),
                           scorer_hidden=int(agent.get("scorer_hidden", 256)))


def modernbert_large(**over: Any) -> EncoderConfig:
    """ModernBERT-large shapes: 28 layers, d 1024, 16 heads x 64, GeGLU 2 x 2624, vocab 50368."""
    v = {"model_type": "modernbert", "vocab_size": 50368, "hidden_size": 1024,
         "num_hidden_layers": 28, "num_attention_heads": 16, "intermediate_size": 2624,
         "global_attn_every_n_layers": 3, "local_attention": 128, "norm_eps": 1e-5,
         "global_rope_theta": 160000.0, "local_rope_theta": 10000.0, "pad_token_id": 50283}
    v.update(over)
    return EncoderConfig.from_value(v)


def large_model(**over: Any) -> ModelConfig:
    return ModelConfig(encoder=modernbert_large(**over))


def small_model() -> ModelConfig:
    """A small config with the same structure (4 layers: global, local, local, global)."""
    enc = EncoderConfig.from_value({
        "model_type": "modernbert", "vocab_size": 512, "hidden_size": 256,
        "num_hidden_layers": 4, "num_attention_heads": 4, "intermediate_size": 384,
        "global_attn_every_n_layers": 3, "local_attention": 16, "pad_token_id": 0})
    return ModelConfig(encoder=enc, head_ffn=512, scorer_hidden=64)
