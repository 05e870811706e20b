"""Which attention layers get the OSCAR INT2 cache.

Same rules as the reference plugin's ``_should_oscar`` / ``_is_hybrid_config``
(``oscar_ascend/plugin.py:184-253``), applied to this framework's layer specs instead
of patched vLLM ``Attention`` modules: a layer is OSCAR when all of

* OSCAR is enabled (``OSCAR_ASCEND_ENABLE`` is not ``0``),
* it is not an MTP (draft) layer - those keep the BF16 shadow cache,
* the model is a hybrid (linear + full attention) model: declared by the model type,
  or else by ``layer_types`` containing both kinds,
* it is a decoder self-attention layer,
* it has no sliding window and no attention sinks.

``heartbeat()`` counts OSCAR attention calls (the reference's liveness counter).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

HYBRID_MODEL_TYPES = {"qwen3_next", "qwen3_5", "qwen3_5_moe", "qwen35", "qwen3_5_text"}

_BEATS = 0


@dataclass
class AttentionSpec:
    layer_id: int
    attn_type: str = "decoder"
    is_mtp: bool = False
    sliding_window: int | None = None
    has_sinks: bool = False


def is_hybrid_config(cfg) -> bool:
    mt = getattr(cfg, "model_type", None)
    if mt in HYBRID_MODEL_TYPES:
        return True
    types = set(getattr(cfg, "layer_types", []) or [])
    return "full_attention" in types and "linear_attention" in types


def oscar_enabled() -> bool:
    return os.environ.get("OSCAR_ASCEND_ENABLE", "auto").strip().lower() not in ("0", "false", "off")


def should_oscar(spec: AttentionSpec, cfg) -> bool:
    return (oscar_enabled() and not spec.is_mtp and is_hybrid_config(cfg) and spec.attn_type == "decoder"
            and spec.sliding_window is None and not spec.has_sinks)


def beat(n: int = 1) -> None:
    global _BEATS
    _BEATS += n


def heartbeat() -> int:
    return _BEATS
