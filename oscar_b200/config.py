"""OSCAR KV-cache configuration, read from the ``OSCAR_ASCEND_*`` environment surface.

The key names, validation rules and derived fields follow the reference plugin
(``oscar_ascend/config.py:35-97``); the defaults are the reference's *serving*
defaults (``delivery/serve_oscar.sh:27-44``): K/V clip 0.96/0.92, sink 128,
recent 256, staging 8192.

Keys that only steered Ascend implementation choices are accepted and validated
but have a fixed meaning here:

* ``OSCAR_ASCEND_USE_TRITON``   – ignored; every GPU op is a hand-written sm_100a kernel.
* ``OSCAR_ASCEND_USE_PAGED``    – ignored; attention always reads INT2 pages in-kernel.
* ``OSCAR_ASCEND_FUSED_PREP``   – ignored; there is no materialised KV to prepare.
* ``OSCAR_ASCEND_PAGED_BLOCK_KV`` – validated against {4,16,32,64,128}, otherwise unused
  (the kernel tile is one 128-token page).
* ``OSCAR_ASCEND_PREFILL_QBLOCK`` – query block of the CPU SDPA oracle (min 128).
* ``OSCAR_ASCEND_PACKED``       – the INT2 pool is always page-packed (17,408 B per
  page and KV head); the MTP draft layer always uses the BF16 shadow pool.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

D_DEFAULT = 256
LEVELS = 4

# Serving defaults (the effective production configuration of the reference).
SERVE_DEFAULTS = {
    "OSCAR_ASCEND_K_CLIP_RATIO": "0.96",
    "OSCAR_ASCEND_V_CLIP_RATIO": "0.92",
    "OSCAR_ASCEND_SINK_TOKENS": "128",
    "OSCAR_ASCEND_RECENT_TOKENS": "256",
    "OSCAR_ASCEND_STAGING_TOKENS": "8192",
    "OSCAR_ASCEND_BATCHED_TOKENS": "15360",
}

_PAGED_BLOCK_KV = (4, 16, 32, 64, 128)


def _env(name: str) -> str | None:
    v = os.environ.get(name)
    if v is None or v.strip() == "":
        return SERVE_DEFAULTS.get(name)
    return v


def _env_int(name: str, default: int) -> int:
    v = _env(name)
    if v is None:
        return default
    try:
        return int(v)
    except ValueError:
        return default


def _env_float(name: str, default: float) -> float:
    v = _env(name)
    if v is None:
        return default
    try:
        return float(v)
    except ValueError:
        return default


def _env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) == "1"


@dataclass
class OscarConfig:
    """Per-layer OSCAR KV settings (one instance per FULL-attention layer group)."""

    head_dim: int = D_DEFAULT
    key_quant_bits: int = 2
    value_quant_bits: int = 2
    k_clip_ratio: float = 0.96
    v_clip_ratio: float = 0.92
    k_rotation_path: str = ""
    v_rotation_path: str = ""
    sink_tokens: int = 128
    recent_tokens: int = 256
    staging_tokens: int = 8192
    # "window": every request has staging rows of its own - its sink pages keep theirs and
    # its recent pages cycle through a small ring - so the sink is never evicted;
    # "hashed": the reference's arena shared by all requests (row = block % rows), whose
    # sink rows are overwritten once a sequence passes staging_tokens.
    staging_layout: str = "window"
    group_size: int = 0
    window_enabled: bool = True
    batched_tokens: int = 15360
    prefill_qblock: int = 512
    paged_block_kv: int = 4
    enable: str = "auto"
    verbose: bool = True
    # Ascend-only switches kept for config compatibility (no effect here).
    use_triton: bool = False
    use_paged: bool = True
    use_fused_prep: bool = False
    packed: bool = True
    extra: dict = field(default_factory=dict)

    @property
    def levels(self) -> int:
        return LEVELS

    @property
    def data_bytes(self) -> int:
        return (self.head_dim * self.key_quant_bits + 7) // 8

    @property
    def slot_bytes(self) -> int:
        """Size of the reference's logical slot (K 96 B + V 64 B at D=256)."""
        return 160

    @property
    def num_groups(self) -> int:
        return 1 if self.group_size == 0 else -(-self.head_dim // self.group_size)

    def clip_index(self, ratio: float) -> int:
        """Ascending-sort index of the clip threshold: ``min(int(ratio*D), D-1)``."""
        return min(int(ratio * self.head_dim), self.head_dim - 1)

    @property
    def enabled(self) -> bool:
        return self.enable != "0"

    def validate(self) -> "OscarConfig":
        if not all(0 <= r <= 1 for r in (self.k_clip_ratio, self.v_clip_ratio)):
            raise ValueError("OSCAR clip ratios must be finite and in [0, 1]")
        if self.group_size != 0:
            raise ValueError("Only per-vector OSCAR quantization (GROUP_SIZE=0) is supported")
        if self.head_dim % 4 != 0:
            raise ValueError(f"head_dim={self.head_dim} must be divisible by 4 for INT2 packing")
        if self.paged_block_kv not in _PAGED_BLOCK_KV:
            raise ValueError("OSCAR_ASCEND_PAGED_BLOCK_KV must be 4, 16, 32, 64 or 128")
        if self.staging_layout not in ("window", "hashed"):
            raise ValueError("OSCAR_STAGING_LAYOUT must be window or hashed")
        self.window_enabled = self.staging_tokens > 0 and (
            self.sink_tokens > 0 or self.recent_tokens > 0
        )
        return self

    @classmethod
    def from_env(cls, head_dim: int | None = None) -> "OscarConfig":
        D = head_dim if head_dim is not None else _env_int("OSCAR_ASCEND_HEAD_DIM", D_DEFAULT)
        cfg = cls(
            head_dim=D,
            k_clip_ratio=_env_float("OSCAR_ASCEND_K_CLIP_RATIO", 0.96),
            v_clip_ratio=_env_float("OSCAR_ASCEND_V_CLIP_RATIO", 0.92),
            k_rotation_path=os.environ.get("OSCAR_ASCEND_K_ROTATION_PATH", ""),
            v_rotation_path=os.environ.get("OSCAR_ASCEND_V_ROTATION_PATH", ""),
            sink_tokens=max(0, _env_int("OSCAR_ASCEND_SINK_TOKENS", 128)),
            recent_tokens=max(0, _env_int("OSCAR_ASCEND_RECENT_TOKENS", 256)),
            staging_tokens=max(0, _env_int("OSCAR_ASCEND_STAGING_TOKENS", 8192)),
            staging_layout=(os.environ.get("OSCAR_STAGING_LAYOUT") or "window").strip().lower(),
            group_size=_env_int("OSCAR_ASCEND_GROUP_SIZE", 0),
            batched_tokens=max(1, _env_int("OSCAR_ASCEND_BATCHED_TOKENS", 15360)),
            prefill_qblock=max(128, _env_int("OSCAR_ASCEND_PREFILL_QBLOCK", 512)),
            paged_block_kv=_env_int("OSCAR_ASCEND_PAGED_BLOCK_KV", 4),
            enable=os.environ.get("OSCAR_ASCEND_ENABLE", "auto"),
            verbose=os.environ.get("OSCAR_ASCEND_VERBOSE", "1") != "0",
            use_triton=_env_flag("OSCAR_ASCEND_USE_TRITON"),
            use_paged=True,
            use_fused_prep=_env_flag("OSCAR_ASCEND_FUSED_PREP"),
            packed=True,
        )
        cfg.extra["enable"] = cfg.enable
        cfg.extra["calib"] = _env_flag("OSCAR_ASCEND_CALIB")
        cfg.extra["calib_token_cap"] = _env_int("OSCAR_ASCEND_CALIB_TOKEN_CAP", 512)
        return cfg.validate()


def profile_settings() -> dict:
    """Diagnostics capture limits (``OSCAR_ASCEND_PROFILE_*``)."""
    steps = _env_int("OSCAR_ASCEND_PROFILE_STEPS", 0)
    min_req = _env_int("OSCAR_ASCEND_PROFILE_MIN_REQUESTS", 0)
    max_tok = _env_int("OSCAR_ASCEND_PROFILE_MAX_TOKENS_PER_REQUEST", 0)
    if min_req < 0 or max_tok < 0:
        raise ValueError("OSCAR diagnostic request filters must be nonnegative")
    return {"steps": steps, "min_requests": min_req, "max_tokens_per_request": max_tok}
