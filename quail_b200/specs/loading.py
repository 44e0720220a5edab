"""Model and device specs as TOML files, the reference's spec format.

Devices (`data/devices/<name>.toml`) give the peaks the planner prices work
against: memory, HBM bandwidth, dense fp8 / bf16 / fp32 / fp4 FLOP/s, SMs,
KV page size, price. Models (`data/models/<name>.toml`) give what the
planner needs of a model without building it: parameters used per token,
layers, widths, heads, weight and KV bytes per element, vocabulary, the
chat turn around prompts. The field names are the reference's
(quail/specs/data/{devices,models}/*.toml, read by
crates/quail-planner/src/cost/specs.rs), so a spec file works in both.

An extension registry can add specs at run time (quail_b200.extensions).
"""

from __future__ import annotations

import os
import tomllib
from dataclasses import dataclass, field, fields

DATA = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data")


@dataclass(frozen=True)
class ModelSpec:
    name: str
    params: float
    layers: int
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    d_head: int
    ffn_width: int
    vocab: int
    w_bytes: float = 1.0
    kv_bytes: float = 2.0
    tied_head: bool = False
    hf_name: str = ""
    revision: str = ""
    w_mem_bytes: float = 0.0
    turn_prefix: str = ""
    turn_suffix: str = ""
    prompt_format: str = ""
    extra: dict = field(default_factory=dict)   # fields this build does not read, kept as written


def _read(path: str) -> dict:
    with open(path, "rb") as f:
        return tomllib.load(f)


def _split(cls, raw: dict) -> dict:
    known = {f.name for f in fields(cls)} - {"extra"}
    out = {k: v for k, v in raw.items() if k in known}
    extra = {k: v for k, v in raw.items() if k not in known}
    if "extra" in {f.name for f in fields(cls)}:
        out["extra"] = extra
    return out


def load_device(path: str):
    from quail_b200.planner.specs import DeviceSpec
    raw = _read(path)
    known = {f.name for f in fields(DeviceSpec)}
    return DeviceSpec(**{k: v for k, v in raw.items() if k in known})


def load_model(path: str) -> ModelSpec:
    return ModelSpec(**_split(ModelSpec, _read(path)))


def _load_dir(kind: str, loader) -> dict:
    d = os.path.join(DATA, kind)
    out = {}
    for name in sorted(os.listdir(d)):
        if name.endswith(".toml"):
            spec = loader(os.path.join(d, name))
            out[spec.name] = spec
    return out


def builtin_devices() -> dict:
    return _load_dir("devices", load_device)


def builtin_models() -> dict:
    return _load_dir("models", load_model)


def model_spec_of(cfg) -> ModelSpec:
    """The spec a decoder config implies (for models without a TOML file)."""
    ffn = 2 * cfg.intermediate
    params = cfg.layers * (cfg.hidden * (cfg.q_dim + 2 * cfg.kv_dim) + cfg.q_dim * cfg.hidden
                           + 3 * cfg.hidden * cfg.intermediate)
    return ModelSpec(name=cfg.name, params=float(params), layers=cfg.layers, hidden=cfg.hidden,
                     num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, d_head=cfg.head_dim,
                     ffn_width=ffn, vocab=cfg.vocab, w_bytes=1.0 if cfg.fp8 else 2.0, tied_head=cfg.tied_head)
