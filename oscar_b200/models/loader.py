"""Hugging Face Qwen3.5 checkpoints (safetensors) into a :class:`HybridModel`.

The target model's weights are published in the Hugging Face layout
(``Qwen3_5ForConditionalGeneration`` / ``Qwen3_5ForCausalLM``; the text tower lives
under ``model.language_model.`` or ``model.``, the MTP head under ``mtp.``).  This
module maps that layout onto the kernels' layout of one tensor-parallel rank:

* every linear becomes a W8A8 :class:`QLinear` - int8 codes, per-output-channel
  symmetric scale ``max|w_row| / 127`` taken over the WHOLE logical row, so a
  row-parallel weight (o_proj / out_proj / down_proj) has the same scale on every rank
  and every TP size holds slices of one quantised model;
* gated attention: ``q_proj`` rows are already per head ``[query | gate]`` (the
  kernels' layout), ``k_proj`` / ``v_proj`` rows follow, one fused ``qkv`` matrix;
* gated DeltaNet: ``in_proj_qkv`` (``[q | k | v]`` over all heads), ``in_proj_z``,
  ``in_proj_b`` and ``in_proj_a`` are regrouped per key head into
  ``[q(dk) k(dk) v(r*dv) z(r*dv)]`` rows followed by ``[b(r) a(r)]`` rows (value head
  ``j`` belongs to key head ``j // r``, as ``repeat_interleave`` in the HF model), then
  zero rows up to a multiple of 8; ``conv1d`` channels keep the ``[q | k | v]`` order
  (this rank's heads of each), the tap order is the same (tap ``K-1`` multiplies the
  current token);
* norms: ``Qwen3_5RMSNorm`` weights are stored as ``w`` and applied as ``1 + w`` by the
  kernels, like the HF model; the gated norm of the DeltaNet multiplies by its weight
  directly, like the HF model;
* the MTP head: ``mtp.fc`` over ``[norm_emb(embed) | norm_hid(hidden)]``,
  ``mtp.pre_fc_norm_embedding`` / ``pre_fc_norm_hidden`` / ``mtp.norm`` and one
  decoder layer ``mtp.layers.0``.

Tensors are read lazily with ``safe_open``; a column-parallel weight reads only this
rank's rows.  The vision tower of the multimodal checkpoints is not used (the framework
serves text).

The reference serves the same checkpoints through its host framework's loader
(``delivery/serve_oscar.sh:76-99`` passes the model directory to ``vllm serve``); the
OSCAR plugin itself adds no weights (``oscar_ascend/backend.py`` quantises only the KV
cache, and the rotations come from ``oscar_rotations.pt``).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

from .config import HybridConfig
from .qwen35 import GDNLayer, FullAttentionLayer, HybridModel, MLP, QLinear, no_random_init

# RoPE scaling fields carried over from a checkpoint's rope_parameters
YARN_KEYS = ("factor", "original_max_position_embeddings", "beta_fast", "beta_slow", "mscale", "mscale_all_dim",
             "attention_factor", "truncate")

# geometry the kernels are built for
KERNEL_HEAD_DIM = 256
KERNEL_LINEAR_HEAD_DIM = 128


class CheckpointError(RuntimeError):
    """The checkpoint does not match the model (missing tensor, wrong shape, unsupported geometry)."""


# ----------------------------------------------------------------------------- config
def _read_json(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


def config_from_hf(source, name: str | None = None) -> HybridConfig:
    """:class:`HybridConfig` of a Hugging Face Qwen3.5 ``config.json`` (a directory, the
    file, or the parsed dict; the multimodal form nests the text model in ``text_config``)."""
    if isinstance(source, dict):
        raw = source
    else:
        path = os.path.join(source, "config.json") if os.path.isdir(source) else source
        raw = _read_json(path)
        name = name or os.path.basename(os.path.dirname(os.path.abspath(path)))
    c = raw.get("text_config") or raw
    if int(c.get("num_experts") or 0) > 0:
        raise CheckpointError("mixture-of-experts checkpoints are not supported (dense SwiGLU MLP only)")
    rope = dict(c.get("rope_parameters") or c.get("rope_scaling") or {})
    theta = rope.get("rope_theta", c.get("rope_theta", 1.0e7))
    partial = rope.get("partial_rotary_factor", c.get("partial_rotary_factor", 0.25))
    kind = rope.get("rope_type", rope.get("type", "default"))
    if kind == "yarn":
        scaling = {k: rope[k] for k in YARN_KEYS if k in rope}
        scaling["rope_type"] = "yarn"
    elif kind in ("default", "mrope", None):
        scaling = None
    else:
        raise CheckpointError(f"unsupported rope scaling {kind!r} (supported: default, yarn)")
    layers = int(c["num_hidden_layers"])
    interval = int(c.get("full_attention_interval", 4))
    types = list(c.get("layer_types") or [])
    cfg = HybridConfig(
        vocab_size=int(c["vocab_size"]), hidden_size=int(c["hidden_size"]),
        intermediate_size=int(c["intermediate_size"]), num_layers=layers, full_attention_interval=interval,
        num_attention_heads=int(c["num_attention_heads"]), num_key_value_heads=int(c["num_key_value_heads"]),
        head_dim=int(c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]),
        partial_rotary_factor=float(partial), rope_theta=float(theta),
        linear_num_key_heads=int(c["linear_num_key_heads"]), linear_num_value_heads=int(c["linear_num_value_heads"]),
        linear_key_head_dim=int(c["linear_key_head_dim"]), linear_value_head_dim=int(c["linear_value_head_dim"]),
        linear_conv_kernel_dim=int(c.get("linear_conv_kernel_dim", 4)), rms_norm_eps=float(c.get("rms_norm_eps", 1e-6)),
        num_mtp_layers=int(c.get("mtp_num_hidden_layers", raw.get("mtp_num_hidden_layers", 0)) or 0),
        max_position=int(c.get("max_position_embeddings", 262144)), name=name or "qwen35-hf", layer_types=types,
        rope_scaling=scaling)
    check_supported(cfg)
    return cfg


def eos_token_ids(path: str) -> list[int]:
    """End-of-sequence token ids of a Hugging Face model directory: ``generation_config.json``
    first, else ``config.json`` (its ``text_config`` too); an int or a list there."""
    for fname in ("generation_config.json", "config.json"):
        f = os.path.join(path, fname)
        if not os.path.exists(f):
            continue
        raw = _read_json(f)
        e = raw.get("eos_token_id", (raw.get("text_config") or {}).get("eos_token_id"))
        if e is not None:
            return [int(e)] if isinstance(e, int) else [int(x) for x in e]
    return []


def generation_defaults(path: str) -> dict:
    """The sampling defaults a checkpoint recommends (``generation_config.json``:
    ``temperature``, ``top_k``, ``top_p``); empty when it recommends none."""
    f = os.path.join(path, "generation_config.json")
    if not os.path.exists(f):
        return {}
    raw = _read_json(f)
    if raw.get("do_sample") is False:
        return {"temperature": 0.0}
    return {k: raw[k] for k in ("temperature", "top_k", "top_p") if raw.get(k) is not None}


def check_supported(cfg: HybridConfig) -> None:
    """Raises :class:`CheckpointError` when the geometry is not one the kernels implement."""
    bad = []
    if cfg.head_dim != KERNEL_HEAD_DIM:
        bad.append(f"head_dim {cfg.head_dim} (kernels: {KERNEL_HEAD_DIM})")
    if cfg.linear_key_head_dim != KERNEL_LINEAR_HEAD_DIM or cfg.linear_value_head_dim != KERNEL_LINEAR_HEAD_DIM:
        bad.append(f"linear head dims {cfg.linear_key_head_dim}/{cfg.linear_value_head_dim} "
                   f"(kernels: {KERNEL_LINEAR_HEAD_DIM})")
    if cfg.linear_conv_kernel_dim != 4:
        bad.append(f"conv kernel {cfg.linear_conv_kernel_dim} (kernels: 4)")
    if cfg.num_attention_heads % cfg.num_key_value_heads or cfg.linear_num_value_heads % cfg.linear_num_key_heads:
        bad.append("query / value heads not a multiple of key heads")
    if len(cfg.layer_types) != cfg.num_layers:
        bad.append(f"{len(cfg.layer_types)} layer types for {cfg.num_layers} layers")
    if bad:
        raise CheckpointError("unsupported model geometry: " + "; ".join(bad))


# ----------------------------------------------------------------------------- tensors
class CheckpointReader:
    """Named tensors of a checkpoint: a directory of ``*.safetensors`` files (sharded with
    ``model.safetensors.index.json`` or not), one file, or a ``{name: tensor}`` dict.
    :meth:`rows` reads only the requested row ranges of a file-backed tensor."""

    def __init__(self, source):
        self._dict = None
        self._files: dict[str, str] = {}
        self._open: dict[str, object] = {}
        if isinstance(source, dict):
            self._dict = source
            return
        if os.path.isdir(source):
            files = sorted(f for f in os.listdir(source) if f.endswith(".safetensors"))
            if not files:
                raise CheckpointError(f"no .safetensors files in {source}")
            paths = [os.path.join(source, f) for f in files]
        else:
            paths = [source]
        from safetensors import safe_open
        for p in paths:
            with safe_open(p, framework="pt") as f:
                for k in f.keys():
                    self._files[k] = p

    def names(self) -> set[str]:
        return set(self._dict) if self._dict is not None else set(self._files)

    def __contains__(self, name: str) -> bool:
        return name in (self._dict if self._dict is not None else self._files)

    def _handle(self, name: str):
        p = self._files[name]
        if p not in self._open:
            from safetensors import safe_open
            self._open[p] = safe_open(p, framework="pt")
        return self._open[p]

    def shape(self, name: str) -> tuple:
        if name not in self:
            raise CheckpointError(f"missing tensor {name}")
        if self._dict is not None:
            return tuple(self._dict[name].shape)
        return tuple(self._handle(name).get_slice(name).get_shape())

    def full(self, name: str) -> torch.Tensor:
        if name not in self:
            raise CheckpointError(f"missing tensor {name}")
        if self._dict is not None:
            return self._dict[name]
        return self._handle(name).get_tensor(name)

    def rows(self, name: str, ranges) -> torch.Tensor:
        """Rows ``[a, b)`` of every range in ``ranges``, concatenated along dim 0."""
        if name not in self:
            raise CheckpointError(f"missing tensor {name}")
        if self._dict is not None:
            t = self._dict[name]
            return torch.cat([t[a:b] for a, b in ranges])
        sl = self._handle(name).get_slice(name)
        return torch.cat([sl[a:b] for a, b in ranges])

    def close(self) -> None:
        self._open.clear()


# ----------------------------------------------------------------------------- quantisation
def quantize_rows(w: torch.Tensor, device) -> QLinear:
    """W8A8 weight of ``w [N, K]``: int8 codes and per-row scale ``max|w_row| / 127``."""
    w = w.to(device=device, dtype=torch.float32)
    s = w.abs().amax(dim=1).clamp_min(1e-12) / 127.0
    q = torch.round(w / s[:, None]).clamp_(-127, 127).to(torch.int8)
    return QLinear(q.contiguous(), s.contiguous())


def quantize_cols(w: torch.Tensor, cols: tuple[int, int], device) -> QLinear:
    """Columns ``[c0, c1)`` of ``w [N, K]`` (a row-parallel shard) with the scale of the whole row."""
    w = w.to(device=device, dtype=torch.float32)
    s = w.abs().amax(dim=1).clamp_min(1e-12) / 127.0
    q = torch.round(w[:, cols[0]:cols[1]] / s[:, None]).clamp_(-127, 127).to(torch.int8)
    return QLinear(q.contiguous(), s.contiguous())


def dequantize(ql: QLinear) -> torch.Tensor:
    return ql.q.float() * ql.s.float()[:, None]


# ----------------------------------------------------------------------------- mapping
@dataclass
class LoadReport:
    loaded: list = field(default_factory=list)      # checkpoint tensors used
    unused: list = field(default_factory=list)      # checkpoint tensors not used (vision tower, ...)
    root: str = ""                                  # text-model prefix found in the checkpoint
    tied_lm_head: bool = False
    mtp_loaded: bool = False


class _Mapper:
    def __init__(self, model: HybridModel, reader: CheckpointReader):
        self.m = model
        self.r = reader
        self.dev = model.device
        self.used: set[str] = set()

    def expect(self, name: str, shape) -> str:
        got = self.r.shape(name)
        if tuple(got) != tuple(shape):
            raise CheckpointError(f"{name}: checkpoint shape {tuple(got)}, model expects {tuple(shape)}")
        self.used.add(name)
        return name

    def vec(self, name: str, n: int) -> torch.Tensor:
        return self.r.full(self.expect(name, (n,))).to(device=self.dev, dtype=torch.float32).contiguous()

    # ---- decoder layer parts
    def norms(self, mixer, pfx: str) -> None:
        H = self.m.cfg.hidden_size
        mixer.input_norm = self.vec(pfx + "input_layernorm.weight", H)
        mixer.post_norm = self.vec(pfx + "post_attention_layernorm.weight", H)

    def attention(self, m: FullAttentionLayer, pfx: str) -> None:
        cfg = self.m.cfg
        H, D = cfg.hidden_size, cfg.head_dim
        nq, nk = cfg.num_attention_heads, cfg.num_key_value_heads
        q = self.expect(pfx + "q_proj.weight", (nq * 2 * D, H))
        k = self.expect(pfx + "k_proj.weight", (nk * D, H))
        v = self.expect(pfx + "v_proj.weight", (nk * D, H))
        o = self.expect(pfx + "o_proj.weight", (H, nq * D))
        kr = [(m.k0 * D, (m.k0 + m.Hk) * D)]
        w = torch.cat([self.r.rows(q, [(m.h0 * 2 * D, (m.h0 + m.Hq) * 2 * D)]), self.r.rows(k, kr),
                       self.r.rows(v, kr)])
        m.qkv = quantize_rows(w, self.dev)
        m.o = quantize_cols(self.r.full(o), (m.h0 * D, (m.h0 + m.Hq) * D), self.dev)
        m.q_norm = self.vec(pfx + "q_norm.weight", D)
        m.k_norm = self.vec(pfx + "k_norm.weight", D)

    def gdn(self, m: GDNLayer, pfx: str) -> None:
        cfg = self.m.cfg
        H = cfg.hidden_size
        nk, nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        dk, dv, r = m.dk, m.dv, m.r
        Kd, Vd = nk * dk, nv * dv
        Kc = cfg.linear_conv_kernel_dim
        qkv = self.expect(pfx + "in_proj_qkv.weight", (2 * Kd + Vd, H))
        z = self.expect(pfx + "in_proj_z.weight", (Vd, H))
        b = self.expect(pfx + "in_proj_b.weight", (nv, H))
        a = self.expect(pfx + "in_proj_a.weight", (nv, H))
        conv = self.expect(pfx + "conv1d.weight", (2 * Kd + Vd, 1, Kc))
        out = self.expect(pfx + "out_proj.weight", (H, Vd))
        parts = []
        for kh in range(m.k0, m.k0 + m.Hk):  # [q k v z] of key head kh and its r value heads
            parts.append(self.r.rows(qkv, [(kh * dk, (kh + 1) * dk), (Kd + kh * dk, Kd + (kh + 1) * dk),
                                           (2 * Kd + kh * r * dv, 2 * Kd + (kh + 1) * r * dv)]))
            parts.append(self.r.rows(z, [(kh * r * dv, (kh + 1) * r * dv)]))
        for kh in range(m.k0, m.k0 + m.Hk):  # [b a] of the value heads of key head kh
            parts.append(self.r.rows(b, [(kh * r, (kh + 1) * r)]))
            parts.append(self.r.rows(a, [(kh * r, (kh + 1) * r)]))
        ql = quantize_rows(torch.cat(parts), self.dev)
        pad = m.inp.q.shape[0] - ql.q.shape[0]
        if pad < 0:
            raise CheckpointError(f"{pfx}: {ql.q.shape[0]} projection rows, model holds {m.inp.q.shape[0]}")
        if pad:
            ql = QLinear(torch.cat([ql.q, ql.q.new_zeros(pad, H)]).contiguous(),
                         torch.cat([ql.s, ql.s.new_ones(pad)]).contiguous())
        m.inp = ql
        w = self.r.full(conv).reshape(2 * Kd + Vd, Kc)
        m.conv_w = torch.cat([w[m.k0 * dk:(m.k0 + m.Hk) * dk], w[Kd + m.k0 * dk:Kd + (m.k0 + m.Hk) * dk],
                              w[2 * Kd + m.v0 * dv:2 * Kd + (m.v0 + m.Hv) * dv]]).to(
            device=self.dev, dtype=torch.float32).contiguous()
        m.A_log = self.vec(pfx + "A_log", nv)[m.v0:m.v0 + m.Hv].contiguous()
        m.dt_bias = self.vec(pfx + "dt_bias", nv)[m.v0:m.v0 + m.Hv].contiguous()
        m.norm_w = self.vec(pfx + "norm.weight", dv)
        m.out = quantize_cols(self.r.full(out), (m.v0 * dv, (m.v0 + m.Hv) * dv), self.dev)

    def mlp(self, mlp: MLP, pfx: str) -> None:
        cfg = self.m.cfg
        H, I = cfg.hidden_size, cfg.intermediate_size
        g = self.expect(pfx + "gate_proj.weight", (I, H))
        u = self.expect(pfx + "up_proj.weight", (I, H))
        d = self.expect(pfx + "down_proj.weight", (H, I))
        rr = [(mlp.i0, mlp.i0 + mlp.I)]
        mlp.gate_up = quantize_rows(torch.cat([self.r.rows(g, rr), self.r.rows(u, rr)]), self.dev)
        mlp.down = quantize_cols(self.r.full(d), (mlp.i0, mlp.i0 + mlp.I), self.dev)


def _find_root(names: set[str]) -> str:
    for root in ("model.language_model.", "model.", ""):
        if root + "embed_tokens.weight" in names:
            return root
    raise CheckpointError("no embed_tokens.weight under model.language_model., model. or the top level")


def load_checkpoint(model: HybridModel, source, strict: bool = True) -> LoadReport:
    """Overwrites ``model``'s weights with the checkpoint's (this rank's slices).

    ``strict``: an MTP head without ``mtp.*`` tensors, or a tensor of a loaded decoder
    layer that the mapping does not use (a bias, say), is an error; otherwise the MTP
    head keeps its weights and such tensors are only reported."""
    reader = source if isinstance(source, CheckpointReader) else CheckpointReader(source)
    try:
        return _load(model, reader, strict)
    finally:
        reader.close()


def _load(model: HybridModel, reader: CheckpointReader, strict: bool) -> LoadReport:
    cfg = model.cfg
    check_supported(cfg)
    names = reader.names()
    rep = LoadReport(root=_find_root(names))
    mp = _Mapper(model, reader)
    root, dev = rep.root, model.device
    H, V = cfg.hidden_size, cfg.vocab_size
    v0 = model.vocab_begin
    v1 = min(V, v0 + model.V_local)
    emb_name = mp.expect(root + "embed_tokens.weight", (V, H))
    emb = torch.zeros(model.V_local, H, dtype=torch.bfloat16, device=dev)
    emb[:v1 - v0] = reader.rows(emb_name, [(v0, v1)]).to(device=dev, dtype=torch.bfloat16)
    model.embed = emb
    head = "lm_head.weight" if "lm_head.weight" in names else None
    if head is None:
        rep.tied_lm_head = True
        head = emb_name
    else:
        mp.expect(head, (V, H))
    model.lm_head = quantize_rows(reader.rows(head, [(v0, v1)]), dev)
    model.final_norm = mp.vec(root + "norm.weight", H)
    for i, (mixer, mlp) in enumerate(model.layers):
        pfx = f"{root}layers.{i}."
        if isinstance(mixer, FullAttentionLayer):
            mp.attention(mixer, pfx + "self_attn.")
        else:
            mp.gdn(mixer, pfx + "linear_attn.")
        mp.norms(mixer, pfx)
        mp.mlp(mlp, pfx + "mlp.")
    if model.mtp is not None:
        if "mtp.fc.weight" in names:
            t = model.mtp
            t.fc = quantize_rows(reader.full(mp.expect("mtp.fc.weight", (H, 2 * H))), dev)
            t.norm_emb = mp.vec("mtp.pre_fc_norm_embedding.weight", H)
            t.norm_hid = mp.vec("mtp.pre_fc_norm_hidden.weight", H)
            t.final_norm = mp.vec("mtp.norm.weight", H)
            mp.attention(t.layer, "mtp.layers.0.self_attn.")
            mp.norms(t.layer, "mtp.layers.0.")
            mp.mlp(t.mlp, "mtp.layers.0.mlp.")
            rep.mtp_loaded = True
        elif strict:
            raise CheckpointError("the model has an MTP head but the checkpoint has no mtp.* tensors "
                                  "(build the model with mtp=False, or load with strict=False)")
    for mixer, _ in model.layers:
        if isinstance(mixer, FullAttentionLayer):
            mixer._split_rotations()
    rep.loaded = sorted(mp.used)
    rep.unused = sorted(names - mp.used)
    if strict:
        pfxs = [f"{root}layers.{i}." for i in range(len(model.layers))]
        if rep.mtp_loaded:
            pfxs.append("mtp.")
        odd = [n for n in rep.unused if any(n.startswith(p) for p in pfxs) and not n.endswith("inv_freq")]
        if odd:
            raise CheckpointError(f"tensors of loaded layers that the mapping does not use: {odd[:6]}")
    return rep


def from_pretrained(path: str, tp=None, device="cpu", oscar=None, kv_mode: str = "int2", rotation: str = "random",
                    mtp: bool = True, num_layers: int | None = None, strict: bool = True,
                    seed: int = 0, config: HybridConfig | None = None) -> HybridModel:
    """A :class:`HybridModel` of this rank holding the checkpoint in ``path`` (a Hugging Face
    model directory: ``config.json`` and ``*.safetensors``).  ``num_layers`` keeps only the
    first layers (testing); the MTP head is built when the config has one and ``mtp``;
    ``seed`` seeds what a checkpoint does not hold (the random KV rotations of
    ``rotation="random"``); ``config`` replaces the checkpoint's ``config.json`` (an
    override such as a RoPE scaling applied to it)."""
    cfg = config if config is not None else config_from_hf(path)
    if num_layers is not None and num_layers < cfg.num_layers:
        cfg = HybridConfig(**{**cfg.to_dict(), "num_layers": num_layers, "layer_types": cfg.layer_types[:num_layers]})
    with no_random_init():
        model = HybridModel(cfg, tp, device=device, seed=seed, oscar=oscar, kv_mode=kv_mode, rotation=rotation,
                            mtp=mtp)
    load_checkpoint(model, path, strict=strict)
    return model


# ----------------------------------------------------------------------------- export
def hf_state_dict(model: HybridModel, dtype=torch.bfloat16, root: str = "model.") -> dict:
    """The inverse mapping: the Hugging Face Qwen3.5 tensors of a single-rank model
    (dequantised W8A8 weights).  Loading the result gives back the same int8 codes and
    scales when ``dtype`` is float32 (bf16 rounds the dequantised weights)."""
    if model.tp.world != 1:
        raise ValueError("export a single-rank (TP1) model")
    cfg = model.cfg
    D, nq, nk = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    out: dict[str, torch.Tensor] = {}

    def put(name, t):
        out[name] = t.detach().to(device="cpu", dtype=dtype).contiguous()

    def attention(m: FullAttentionLayer, pfx):
        w = dequantize(m.qkv)
        put(pfx + "q_proj.weight", w[:nq * 2 * D])
        put(pfx + "k_proj.weight", w[nq * 2 * D:nq * 2 * D + nk * D])
        put(pfx + "v_proj.weight", w[nq * 2 * D + nk * D:])
        put(pfx + "o_proj.weight", dequantize(m.o))
        put(pfx + "q_norm.weight", m.q_norm)
        put(pfx + "k_norm.weight", m.k_norm)

    def gdn(m: GDNLayer, pfx):
        dk, dv, r = m.dk, m.dv, m.r
        w = dequantize(m.inp)
        grp = 2 * dk + 2 * r * dv
        g = w[:m.Hk * grp].view(m.Hk, grp, -1)
        ba = w[m.n_qkvz:m.n_qkvz + m.n_ba].view(m.Hk, 2 * r, -1)
        H = w.shape[1]
        put(pfx + "in_proj_qkv.weight", torch.cat([g[:, :dk].reshape(-1, H), g[:, dk:2 * dk].reshape(-1, H),
                                                   g[:, 2 * dk:2 * dk + r * dv].reshape(-1, H)]))
        put(pfx + "in_proj_z.weight", g[:, 2 * dk + r * dv:].reshape(-1, H))
        put(pfx + "in_proj_b.weight", ba[:, :r].reshape(-1, H))
        put(pfx + "in_proj_a.weight", ba[:, r:].reshape(-1, H))
        put(pfx + "conv1d.weight", m.conv_w.unsqueeze(1))
        put(pfx + "A_log", m.A_log)
        put(pfx + "dt_bias", m.dt_bias)
        put(pfx + "norm.weight", m.norm_w)
        put(pfx + "out_proj.weight", dequantize(m.out))

    def mlp(ml: MLP, pfx):
        w = dequantize(ml.gate_up)
        put(pfx + "gate_proj.weight", w[:ml.I])
        put(pfx + "up_proj.weight", w[ml.I:])
        put(pfx + "down_proj.weight", dequantize(ml.down))

    def layer(mixer, ml, pfx):
        if isinstance(mixer, FullAttentionLayer):
            attention(mixer, pfx + "self_attn.")
        else:
            gdn(mixer, pfx + "linear_attn.")
        put(pfx + "input_layernorm.weight", mixer.input_norm)
        put(pfx + "post_attention_layernorm.weight", mixer.post_norm)
        mlp(ml, pfx + "mlp.")

    put(root + "embed_tokens.weight", model.embed[:cfg.vocab_size].float())
    put("lm_head.weight", dequantize(model.lm_head))
    put(root + "norm.weight", model.final_norm)
    for i, (mixer, ml) in enumerate(model.layers):
        layer(mixer, ml, f"{root}layers.{i}.")
    if model.mtp is not None:
        t = model.mtp
        put("mtp.fc.weight", dequantize(t.fc))
        put("mtp.pre_fc_norm_embedding.weight", t.norm_emb)
        put("mtp.pre_fc_norm_hidden.weight", t.norm_hid)
        put("mtp.norm.weight", t.final_norm)
        layer(t.layer, t.mlp, "mtp.layers.0.")
    return out


def hf_config(cfg: HybridConfig) -> dict:
    """A Hugging Face ``Qwen3_5TextConfig``-style ``config.json`` dict of ``cfg``."""
    return {
        "model_type": "qwen3_5_text", "architectures": ["Qwen3_5ForCausalLM"],
        "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size, "intermediate_size": cfg.intermediate_size,
        "num_hidden_layers": cfg.num_layers, "full_attention_interval": cfg.full_attention_interval,
        "layer_types": list(cfg.layer_types), "num_attention_heads": cfg.num_attention_heads,
        "num_key_value_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim,
        "linear_num_key_heads": cfg.linear_num_key_heads, "linear_num_value_heads": cfg.linear_num_value_heads,
        "linear_key_head_dim": cfg.linear_key_head_dim, "linear_value_head_dim": cfg.linear_value_head_dim,
        "linear_conv_kernel_dim": cfg.linear_conv_kernel_dim, "rms_norm_eps": cfg.rms_norm_eps,
        "max_position_embeddings": cfg.max_position, "mtp_num_hidden_layers": cfg.num_mtp_layers,
        "hidden_act": "silu", "tie_word_embeddings": False,
        "rope_parameters": {"rope_type": "default", "rope_theta": cfg.rope_theta,
                            "partial_rotary_factor": cfg.partial_rotary_factor, "mrope_section": [11, 11, 10],
                            "mrope_interleaved": True, **(cfg.rope_scaling or {})},
    }


def save_hf_checkpoint(model: HybridModel, path: str, dtype=torch.bfloat16, max_shard_bytes: int = 4 << 30) -> None:
    """Writes ``model`` (TP1) as a Hugging Face model directory: ``config.json``,
    ``model-XXXXX-of-YYYYY.safetensors`` shards and ``model.safetensors.index.json``."""
    from safetensors.torch import save_file
    sd = hf_state_dict(model, dtype=dtype)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config(model.cfg), f, indent=2)
    shards, cur, size = [], {}, 0
    for name in sorted(sd):
        nbytes = sd[name].numel() * sd[name].element_size()
        if cur and size + nbytes > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[name] = sd[name]
        size += nbytes
    shards.append(cur)
    index = {}
    for i, shard in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(shard, os.path.join(path, fname), metadata={"format": "pt"})
        index.update({k: fname for k in shard})
    total = sum(t.numel() * t.element_size() for t in sd.values())
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": index}, f, indent=2)
