"""The engine configuration a session runs on.

Same fields as the reference's EngineConfig (quail/api/config.py:21-42):
`model` and `device` name the weights and the hardware, `gpus` counts model
copies on one host (1, 2, 4 or 8), `gpu_timing` records a CUDA event pair
per forward chunk, `canvas_draws` and `attention` are kept for API parity.
Additions: `weights`, a directory of HF safetensors to load instead of
random-init weights of the named architecture; `parallel`, how each model
copy spreads over GPUs ("dp": one GPU per copy; "tp": tensor-parallel
copies; "ep": expert-parallel copies of a mixture-of-experts model); and
`group_gpus`, the GPUs of one tp / ep copy (default: all `gpus`, one copy).
Rows are sharded over the copies either way.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class Refusal:
    reasons: tuple
    constraint: str
    needed: float = 1
    available: float = 0
    unit: str = ""


class RefusalError(RuntimeError):
    """The planner refuses to run a query or configuration, and says why."""

    def __init__(self, refusal: Refusal):
        self.refusal = refusal
        super().__init__("; ".join(refusal.reasons))


DEVICES = ("b200", "cpu")


@dataclass(frozen=True, kw_only=True)
class EngineConfig:
    model: str
    device: str
    gpus: int = 1
    backend: str = "quail"
    gpu_timing: bool = False
    canvas_draws: int = 4
    attention: str | None = None
    weights: str | None = None
    parallel: str = "dp"
    group_gpus: int | None = None   # GPUs per tp / ep model copy (None: every GPU, one copy)
    chunk_tokens: int | None = None
    tokenizer: str | None = None   # a tokenizer.json (or its directory), or "words" / "bytes"
    seed: int = 0
    extra: dict = field(default_factory=dict)


def resolve_model(name: str, registry=None):
    from quail_b200.models.config import MODEL_CONFIGS
    if registry is not None:
        found = registry.model(name)
        if found is not None:
            return found
    if name in MODEL_CONFIGS:
        return MODEL_CONFIGS[name]
    names = registry.model_names() if registry is not None else sorted(MODEL_CONFIGS)
    return Refusal(reasons=(f"unknown model {name!r}; registered models: {names}",),
                   constraint="unknown_model", needed=1, available=0, unit="specs")


def check_config(config: EngineConfig, registry=None):
    """The decoder config a session runs, or a RefusalError naming what cannot run.

    `registry` (quail_b200.extensions.ExtensionRegistry) adds models to the built-in ones.
    """
    model = resolve_model(config.model, registry)
    if isinstance(model, Refusal):
        raise RefusalError(model)
    if config.device not in DEVICES:
        raise RefusalError(Refusal(reasons=(f"unknown device {config.device!r}; devices: {list(DEVICES)}",),
                                   constraint="unknown_device"))
    if config.backend != "quail" and (registry is None or registry.backend(config.backend) is None):
        raise RefusalError(Refusal(reasons=(f"unknown backend {config.backend!r}",), constraint="unknown_backend"))
    if config.gpus not in (1, 2, 4, 8):
        raise RefusalError(Refusal(reasons=(f"gpus must be 1, 2, 4 or 8, not {config.gpus}",),
                                   constraint="unsupported_backend_configuration"))
    if config.attention not in (None, "tree", "unified"):
        raise RefusalError(Refusal(reasons=("attention is 'tree', 'unified' or None",),
                                   constraint="unsupported_backend_configuration"))
    # what each split of a model over several GPUs runs on (backends/quail/backend.py:18-88 is the
    # reference's supports(): device, architecture, gpus)
    if config.parallel not in ("dp", "tp", "ep"):
        raise RefusalError(Refusal(reasons=(f"parallel is 'dp', 'tp' or 'ep', not {config.parallel!r}",),
                                   constraint="unsupported_backend_configuration"))
    if config.parallel == "tp" and (model.is_hybrid or model.is_moe or model.role != "generative"):
        raise RefusalError(Refusal(reasons=(f"tensor parallelism runs dense Qwen3 decoders, not {model.name!r}",),
                                   constraint="unsupported_backend_configuration"))
    if config.parallel == "ep" and not model.is_moe:
        raise RefusalError(Refusal(reasons=(f"expert parallelism needs a mixture-of-experts model, not {model.name!r}",),
                                   constraint="unsupported_backend_configuration"))
    if config.parallel != "dp":
        g = group_size(config)
        if config.device == "cpu" and config.gpus > 1:
            raise RefusalError(Refusal(reasons=(f"{config.parallel} copies run on GPUs, not the CPU",),
                                       constraint="unsupported_backend_configuration"))
        if g not in (1, 2, 4, 8) or config.gpus % g:
            raise RefusalError(Refusal(
                reasons=(f"group_gpus={g} must be 1, 2, 4 or 8 and divide gpus={config.gpus}",),
                constraint="unsupported_backend_configuration"))
        if config.parallel == "tp" and (model.num_q_heads % g or model.num_kv_heads % g
                                        or model.intermediate % (g * 128)):
            raise RefusalError(Refusal(
                reasons=(f"{model.name} does not split over {g} GPUs: its q heads ({model.num_q_heads}), kv heads "
                         f"({model.num_kv_heads}) and MLP width / 128 ({model.intermediate // 128}) must divide",),
                constraint="unsupported_backend_configuration"))
        if config.parallel == "ep" and model.num_experts % g:
            raise RefusalError(Refusal(
                reasons=(f"{model.num_experts} experts do not split over {g} GPUs",),
                constraint="unsupported_backend_configuration"))
    return model


def group_size(config: EngineConfig) -> int:
    """GPUs of one model copy: 1 for data parallelism, else group_gpus (default: all gpus)."""
    if config.parallel == "dp":
        return 1
    return config.group_gpus or config.gpus
