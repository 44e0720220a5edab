"""Per-session registry of models, devices and logical rules.

`ExtensionRegistry` lets a session run a model or price a device that the
built-in specs do not list, and add a rule that rewrites a query's syntax
tree before it runs (for example a site-specific default HINT):

    reg = built_in_registry()
    reg.register_model("my-qwen3-1b", QWEN3_06B.with_(name="my-qwen3-1b", layers=20))
    reg.register_device(DeviceSpec("my-gpu", mem_bytes=..., ...))
    reg.register_rule("no-limit", lambda tree: tree)
    Session(EngineConfig(model="my-qwen3-1b", device="cpu"), registry=reg)

Lookups fall back to the built-in registry (models/config.py, the TOML
specs). Reference: quail/extensions.py (per-session registries of models,
devices, backends, runtimes and rules) and quail/builtins.py.
"""

from __future__ import annotations

from collections.abc import Callable


class ExtensionRegistry:
    def __init__(self, parent: "ExtensionRegistry | None" = None):
        self.parent = parent
        self.models: dict = {}
        self.devices: dict = {}
        self.rules: dict[str, Callable[[dict], dict]] = {}
        self.backends: dict[str, Callable] = {}

    # models ---------------------------------------------------------
    def register_model(self, name: str, config) -> None:
        """A decoder config (quail_b200.models.config.DecoderConfig) under an EngineConfig model name."""
        if name in self.models:
            raise ValueError(f"model {name!r} is already registered")
        self.models[name] = config

    def model(self, name: str):
        if name in self.models:
            return self.models[name]
        return self.parent.model(name) if self.parent is not None else None

    def model_names(self) -> list[str]:
        own = set(self.models)
        return sorted(own | set(self.parent.model_names() if self.parent is not None else ()))

    # devices --------------------------------------------------------
    def register_device(self, spec) -> None:
        """A planner DeviceSpec (quail_b200.planner.specs)."""
        if spec.name in self.devices:
            raise ValueError(f"device {spec.name!r} is already registered")
        self.devices[spec.name] = spec

    def device(self, name: str):
        if name in self.devices:
            return self.devices[name]
        return self.parent.device(name) if self.parent is not None else None

    # backends -------------------------------------------------------
    def register_backend(self, name: str, factory: Callable) -> None:
        """An engine other than this one's (factory(config, registry) -> an object with run_region),
        named by EngineConfig.backend; `quail_b200.baselines.register_baselines` adds "vllm"."""
        if name == "quail" or name in self.backends:
            raise ValueError(f"backend {name!r} is already registered")
        self.backends[name] = factory

    def backend(self, name: str):
        if name in self.backends:
            return self.backends[name]
        return self.parent.backend(name) if self.parent is not None else None

    # logical rules --------------------------------------------------
    def register_rule(self, name: str, rule: Callable[[dict], dict]) -> None:
        """A rewrite of a query's syntax tree (the parser's JSON), run before planning."""
        self.rules[name] = rule

    def apply_rules(self, tree: dict) -> dict:
        if self.parent is not None:
            tree = self.parent.apply_rules(tree)
        for rule in self.rules.values():
            tree = rule(tree)
        return tree


class _BuiltIns(ExtensionRegistry):
    def model(self, name: str):
        from quail_b200.models.config import MODEL_CONFIGS
        return MODEL_CONFIGS.get(name)

    def model_names(self) -> list[str]:
        from quail_b200.models.config import MODEL_CONFIGS
        return sorted(MODEL_CONFIGS)

    def device(self, name: str):
        from quail_b200.planner.specs import DEVICES
        return DEVICES.get(name)


def built_in_registry() -> ExtensionRegistry:
    """A registry that answers with the built-in models and devices, and can take more."""
    return ExtensionRegistry(parent=_BuiltIns())
