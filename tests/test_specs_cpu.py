"""TOML specs and the extension registry.

The spec files use the reference's field names (quail/specs/data/{devices,
models}/*.toml); every model spec must agree with the architecture this
build runs under that name, and the registry must let a session run a model
and price a device the built-ins do not list.
"""

import pyarrow as pa
import pytest

import quail_b200 as quail
from quail_b200.extensions import built_in_registry
from quail_b200.models.config import MODEL_CONFIGS, QWEN3_TINY
from quail_b200.planner.budgets import Budgets
from quail_b200.planner.specs import DEVICES, DeviceSpec
from quail_b200.specs.loading import builtin_devices, builtin_models


def test_the_four_devices_load_with_their_peaks():
    devs = builtin_devices()
    assert set(devs) == {"b200", "h100-sxm", "l40s", "rtx-pro-6000-blackwell-server"}
    assert devs["b200"].fp8_flops == 4.5e15 and devs["b200"].page_tokens == 128 and devs["b200"].sms == 148
    assert devs["h100-sxm"].bf16_flops < devs["b200"].bf16_flops
    assert DEVICES["l40s"].mem_bytes < DEVICES["h100-sxm"].mem_bytes
    # the planner prices on any of them
    for name in devs:
        b = Budgets.for_model(MODEL_CONFIGS["qwen3-4b-fp8"], name)
        assert b.chunk_tokens > 0 and b.pass_seconds(16384, 200) > 0


@pytest.mark.parametrize("name", sorted(builtin_models()))
def test_model_specs_agree_with_the_architectures(name):
    spec = builtin_models()[name]
    cfg = MODEL_CONFIGS[name]
    assert (spec.layers, spec.hidden, spec.num_q_heads, spec.num_kv_heads, spec.d_head, spec.vocab) == \
        (cfg.layers, cfg.hidden, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.vocab)
    assert spec.tied_head == cfg.tied_head
    assert spec.params > 0 and spec.w_bytes in (0.5, 1.0, 2.0)


def test_a_registered_model_runs_and_a_registered_device_prices():
    reg = built_in_registry()
    reg.register_model("my-tiny", QWEN3_TINY.with_(name="my-tiny", layers=1))
    reg.register_device(DeviceSpec("my-gpu", mem_bytes=24e9, hbm_bw=1e12, fp8_flops=0.5e15, bf16_flops=0.25e15))
    with pytest.raises(ValueError):
        reg.register_model("my-tiny", QWEN3_TINY)
    assert reg.model("qwen3-4b-fp8") is MODEL_CONFIGS["qwen3-4b-fp8"]      # built-ins still answer
    assert reg.device("my-gpu").hbm_bw == 1e12
    cfg = quail.EngineConfig(model="my-tiny", device="cpu", chunk_tokens=256)
    with pytest.raises(quail.RefusalError):
        quail.Session(config=cfg)                                          # unknown without the registry
    with quail.Session(config=cfg, registry=reg) as s:
        s.register("t", pa.table({"id": [0, 1, 2], "body": ["a cat", "a dog", "a fish"]}))
        out = s.sql("SELECT id, AI.SCORE(PROMPT('Is it a pet? {0}', body)) AS s FROM t").collect()
        assert out.num_rows == 3 and all(0 <= v <= 1 for v in out.column("s").to_pylist())
        assert s.engine().cfg.layers == 1
    assert Budgets.for_model(QWEN3_TINY, "my-gpu", registry=reg).device.name == "my-gpu"


def test_a_registered_rule_rewrites_the_query():
    reg = built_in_registry()

    def at_most_two(tree):
        if tree.get("type") == "select" and tree.get("limit") is None:
            tree = dict(tree, limit={"type": "literal", "kind": "int", "value": 2})
        return tree
    reg.register_rule("at-most-two", at_most_two)
    with quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu"), registry=reg) as s:
        s.register("t", pa.table({"id": [0, 1, 2, 3]}))
        assert s.sql("SELECT id FROM t").collect().num_rows == 2


def test_public_names_and_the_bigquery_dialect():
    import quail
    for name in ("ColumnRef", "ExtensionRegistry", "PhysicalGraph", "PhysicalNode", "ExtensionNode", "SQLDialect",
                 "lower_prompt", "QueryRun", "QueryStatus", "QueryFailedError", "SHARED_PRE"):
        assert hasattr(quail, name), name
    assert quail.ColumnRef.parse("t.body") == quail.ColumnRef("body", "t")
    lowered = quail.lower_prompt(quail.bind_prompt("Is it {0}?"), _Words())
    assert lowered.around([7, 8])[len(lowered.preamble):len(lowered.preamble) + 2] == [7, 8]
    with quail.Session(config=quail.EngineConfig(model="qwen3-tiny", device="cpu")) as s:
        s.register("reviews", pa.table({"id": [1, 2, 3], "my col": ["a", "b", "c"]}))
        bq = s.sql("SELECT id, `my col` FROM `proj.ds.reviews` WHERE SAFE_CAST(id AS INT) > 1 "
                   "AND `my col` <> 'it''s `x`'", dialect="bq").collect()
        assert bq.column("id").to_pylist() == [2, 3]
        s.sql("SET datafusion.sql_parser.dialect = 'BigQuery'").run()
        assert s.sql("SELECT id FROM `reviews`").collect().num_rows == 3
    assert quail.SQLDialect.of("BigQuery") is quail.SQLDialect.BQ


class _Words:
    def encode(self, text):
        return [hash(w) % 1000 for w in text.split()]
