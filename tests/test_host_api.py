"""Host-side contracts of the drop-in API (no GPU needed).

Restates the reference's frontend / cache / selection host tests
(test/python/test_frontend.py, test_cache_adversarial.py,
test_selection.py) for this build.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from ragged import (ArtifactCache, CacheMismatch, CompilationError, Compiler, Hints, Optimizations, ProgramSpec,
                    SpecializationLimit, ValidationError)
from ragged import selection, workloads
from ragged.compiler import schedules_for


@pytest.mark.parametrize("kwargs,match", [
    (dict(op="mean"), "op must"), (dict(op="sum", dtype="f16"), "dtype"), (dict(op="sum", feature_dim=0), "feature_dim"),
    (dict(op="sum", feature_dim=1025), "feature_dim"), (dict(op="sum", offsets_dtype="u32"), "offsets_dtype"),
    (dict(op="sum", strategy="fast"), "strategy"), (dict(op="sum", alias="inplace"), "in-place"),
    (dict(op="sum", chip="sm_89"), "chip"), (dict(op="max", mask=True), "mask"),
    (dict(op="sum", scale=float("inf")), "scale")])
def test_spec_validation(kwargs, match):
    with pytest.raises(ValidationError, match=match):
        ProgramSpec(**kwargs)


def test_hints_and_optimizations_validation():
    with pytest.raises(ValidationError):
        Hints(max_len=-1)
    with pytest.raises(ValidationError):
        Hints(min_len=5, max_len=4)
    with pytest.raises(ValidationError):
        Optimizations(vectorize=1)
    with pytest.raises(ValidationError):
        Optimizations(feature_tile=3)


@pytest.mark.parametrize("d,dtype,expected", [(128, "f32", (32, 4)), (128, "bf16", (16, 8)), (1, "f32", (1, 1)),
                                              (2, "f32", (1, 2)), (3, "bf16", (4, 1)), (1024, "f32", (32, 4)),
                                              (100, "f32", (32, 4)), (256, "bf16", (32, 8))])
def test_geometry(d, dtype, expected):
    assert Optimizations().geometry(d, dtype) == expected


def test_spec_roundtrip_and_hash():
    spec = ProgramSpec("softmax", "bf16", 128, "i64", hints=Hints(max_len=7))
    assert ProgramSpec.from_dict(spec.to_dict()) == spec
    assert spec.ir_hash != ProgramSpec("softmax", "bf16", 128, "i32").ir_hash
    assert spec.signature == "softmax:bf16:D128:i64:sm_100a"


def test_compile_cache_hit_and_adaptive(tmp_path, native_library):
    cache = ArtifactCache(tmp_path)
    spec = ProgramSpec("sum", "f32", 128)
    first = Compiler().compile(spec, cache)
    second = Compiler().compile(spec, cache)
    assert not first.cache_hit and second.cache_hit
    assert second.schedules == first.schedules
    naive = Compiler().compile(ProgramSpec("sum", "f32", 128, strategy="naive"), cache)
    assert naive.schedules == ("naive",) and not naive.selects


def test_unsupported_features_fail_to_compile(tmp_path, native_library):
    cache = ArtifactCache(tmp_path)
    with pytest.raises(CompilationError, match="not implemented"):
        Compiler().compile(ProgramSpec("sum", debug_visits=True), cache)


def test_mask_scale_and_inplace_specialisations_compile(tmp_path, native_library):
    cache = ArtifactCache(tmp_path)
    for spec in (ProgramSpec("softmax", mask=True), ProgramSpec("softmax", alias="inplace"),
                 ProgramSpec("softmax", mask=True, scale=0.5, alias="inplace"), ProgramSpec("sum", scale=2.0),
                 ProgramSpec("max", "bf16", 8, scale=-1.5)):
        program = Compiler().compile(spec, cache)
        assert program.spec == spec


def test_cache_rejects_tampering_and_limits(tmp_path, native_library):
    cache = ArtifactCache(tmp_path, max_specializations=2)
    Compiler().compile(ProgramSpec("sum", "f32", 8, strategy="naive"), cache)
    Compiler().compile(ProgramSpec("sum", "f32", 8, hints=Hints(max_len=3), strategy="naive"), cache)
    with pytest.raises(SpecializationLimit):
        Compiler().compile(ProgramSpec("sum", "f32", 8, hints=Hints(max_len=4), strategy="naive"), cache)
    ledger_path = next(tmp_path.glob("ledger-*.json"))
    ledger = json.loads(ledger_path.read_text())
    for record in ledger["records"].values():
        record["metadata"]["schedules"] = ["rowbalanced"]
    ledger_path.write_text(json.dumps(ledger))
    with pytest.raises(CacheMismatch, match="SHA256"):
        Compiler().compile(ProgramSpec("sum", "f32", 8, hints=Hints(max_len=3), strategy="naive"), cache)
    ledger["library_sha256"] = "0" * 64
    ledger_path.write_text(json.dumps(ledger))
    with pytest.raises(CacheMismatch, match="another library build"):
        Compiler().compile(ProgramSpec("sum", "f32", 8, strategy="naive"), cache)


def test_cache_ledger_survives_concurrent_publishers(tmp_path, native_library):
    """Processes publishing different specializations into one ledger at
    once: every record lands (the flock + re-read + atomic replace)."""
    import multiprocessing
    context = multiprocessing.get_context("spawn")
    with context.Pool(4) as pool:
        pool.starmap(_publish_one, [(str(tmp_path), d) for d in range(1, 13)])
    cache = ArtifactCache(tmp_path)
    for d in range(1, 13):
        assert Compiler().compile(ProgramSpec("max", "f32", d, strategy="naive"), cache).cache_hit


def _publish_one(root, d):
    import sys
    sys.path[:0] = [str(Path(__file__).resolve().parents[1] / "ragged-mlir_b200")]
    from ragged import ArtifactCache as Cache, Compiler as Comp, ProgramSpec as Spec
    Comp().compile(Spec("max", "f32", d, strategy="naive"), Cache(root))


def test_schedules_for():
    assert schedules_for(ProgramSpec("sum", strategy="naive")) == ["naive"]
    assert schedules_for(ProgramSpec("sum", optimizations=Optimizations(classification=False))) == ["naive"]


def test_cost_model_terms_and_choice():
    terms = selection.features(n=2**18, b=1000, d=1, max_len=4000, span=1, element_bytes=4, op="sum", l2_mib=1.0)
    assert terms[0] == 1.0 and terms[1] == 1.0 and terms[3] == 1.0
    assert terms[4] == pytest.approx(np.log2(4000 * 1000 / 2**18))
    assert terms[5] == pytest.approx(1.0 + 1000 * 4 / 2**20 - 1.0)
    model = selection.CostModel.from_dict({
        "version": 3, "margin": 0.1, "l2_mib": 100.0,
        "coefficients": {"reduce": {"rowbalanced": [10, 0, 0, 0, 0, 0], "naive": [5, 0, 0, 0, 0, 0]},
                         "softmax": {"classified": [10, 0, 0, 0, 0, 0], "naive": [9.5, 0, 0, 0, 0, 0]}}})
    assert model.choose("sum", 100, 10, 4, None, 4)[0] == "rowbalanced"     # no length statistics
    assert model.choose("sum", 100, 10, 4, 50, 4)[0] == "naive"            # 5 < 10 * 0.9
    assert model.choose("softmax", 100, 10, 4, 50, 4)[0] == "classified"   # 9.5 is within the margin
    with pytest.raises(CacheMismatch):
        selection.CostModel.from_dict({"version": 3, "margin": 0.0, "l2_mib": 1.0,
                                       "coefficients": {"reduce": {"rowbalanced": [-1] * 6},
                                                        "softmax": {"classified": [0] * 6}}})


def test_shipped_cost_model_loads():
    model = selection.default_model()
    assert set(model.coefficients) == {"reduce", "softmax"}
    assert model.chooser is not None and set(model.chooser.classes) == {"classified", "naive", "rowbalanced"}
    assert model.calibration["heldout_share"] >= 0.9  # the calibration run's held-out group (B200)


def _chooser_dict(**overrides):
    """Three one-split trees: naive scores +1 when log2(N) <= 10, else -1;
    the other schedules score 0 (one leaf each)."""
    data = {"features": selection.CHOICE_FEATURES, "classes": ["classified", "naive", "rowbalanced"],
            "baseline": [0.0, 0.0, 0.0],
            "nodes": {"feature": [0, 0, 0, 0, 0], "threshold": [0.0, 10.0, 0.0, 0.0, 0.0],
                      "left": [-1, 2, -1, -1, -1], "right": [-1, 3, -1, -1, -1],
                      "value": [0.0, 0.0, 1.0, -1.0, 0.0], "leaf": [True, False, True, True, True]},
            "roots": [0, 1, 4], "tree_class": [0, 1, 2], "max_depth": 1}
    data.update(overrides)
    return data


def test_tree_scores_in_the_library_match_the_numpy_walk():
    """rg_tree_scores (C, used by choose) and TreeChooser.scores (NumPy) give
    identical scores for the shipped model on calibration cases, and the C
    walk rejects out-of-range nodes instead of reading past the arrays."""
    import json
    from ragged import _native
    from ragged.errors import ValidationError
    model = selection.default_model()
    chooser = model.chooser
    data = json.loads((Path(selection.__file__).parent / "calibration" / "b200.json").read_text())
    for case in data["cases"][::37]:
        x = selection.choice_features(case["op"], case["n"], case["b"], case["d"], case["max_len"],
                                      4 if case["dtype"] == "f32" else 2)
        assert np.array_equal(chooser.fast_scores(x), chooser.scores(x))
    toy = selection.TreeChooser.from_dict(_chooser_dict())
    broken = {k: v for k, v in toy.native_arrays.items() if k != "_args"}
    broken["left"] = np.array([-1, 9, -1, -1, -1], dtype=np.int32)
    with pytest.raises(ValidationError, match="out of range"):
        _native.tree_scores(broken, selection.choice_features("sum", 512, 4, 8, 128, 4), 3, toy.max_depth)


def test_tree_chooser_choice_and_validation():
    linear = {"reduce": {s: [10, 0, 0, 0, 0, 0] for s in ("classified", "naive", "rowbalanced")},
              "softmax": {s: [10, 0, 0, 0, 0, 0] for s in ("classified", "naive")}}
    model = selection.CostModel.from_dict({"version": 4, "margin": 0.0, "l2_mib": 100.0, "coefficients": linear,
                                           "chooser": _chooser_dict()})
    assert model.choose("sum", 512, 4, 8, 128, 8)[0] == "naive"            # log2(512) = 9 <= 10
    choice, details = model.choose("sum", 1 << 20, 4, 8, 128, 8)
    assert choice == "rowbalanced" and details["scores"]["naive"] == -1.0  # ties go to the family default
    assert model.choose("softmax", 1 << 20, 4, 8, 128, 8)[0] == "classified"
    assert model.choose("sum", 512, 4, 8, None, 8)[0] == "rowbalanced"     # no length statistics
    assert model.choose("sum", 512, 4, 8, 128, 8, available=("classified", "rowbalanced"))[0] == "rowbalanced"
    checks = [list(selection.choice_features("sum", 512, 4, 8, 128, 4)) + ["naive"]]
    selection.TreeChooser.from_dict(_chooser_dict(checks=checks))
    bad = [
        _chooser_dict(checks=[checks[0][:-1] + ["classified"]]),               # recorded choice not reproduced
        _chooser_dict(features="other"),
        _chooser_dict(classes=["classified", "naive", "naive"]),
        _chooser_dict(roots=[0, 1, 9]),
        _chooser_dict(nodes={**_chooser_dict()["nodes"], "left": [-1, 7, -1, -1, -1]}),
        _chooser_dict(nodes={**_chooser_dict()["nodes"], "feature": [0, 99, 0, 0, 0]}),
        _chooser_dict(baseline=[0.0, 0.0]),
    ]
    for data in bad:
        with pytest.raises(CacheMismatch):
            selection.TreeChooser.from_dict(data)
    with pytest.raises(CacheMismatch):
        selection.CostModel.from_dict({"version": 4, "margin": 0.0, "l2_mib": 1.0, "coefficients": linear})


@pytest.mark.parametrize("name", workloads.CONFIGS)
def test_workload_generators(name):
    w = workloads.make(name, scale=0.01)
    offsets = w.offsets()
    assert offsets[0] == 0 and offsets[-1] == w.n and np.all(np.diff(offsets.astype(np.int64)) >= 0)
    values = w.host_values(slice(0, 100))
    assert values.shape == (min(100, w.n), w.d)


def test_full_size_workloads_match_configuration():
    assert workloads.make("c1").n == 1_058_479
    c2 = workloads.make("c2_max")
    assert c2.n == 12_800_000 and c2.b == 200_000 and int((c2.lengths == 0).sum()) == 2000
    c5 = workloads.make("c5")
    assert c5.n == 200_000_000 and c5.b == 4_000_000 and c5.lengths.max() == 50_000_000
    assert int((c5.lengths > c5.n // 8).sum()) == 3


def test_report_says_which_optimisation_controls_had_an_effect():
    effects = Optimizations(shuffle=False, feature_tile=8).effects()
    assert effects["applied"] == ["classification", "vectorize"]
    assert {"shuffle", "online_fusion", "warp_mapping", "feature_tile", "pointwise_fusion"} <= set(effects["no_effect"])
    assert "pointwise_fusion" in Optimizations().effects(transformed=True)["applied"]
    every = set(effects["applied"]) | set(effects["no_effect"])
    assert every == {"classification", "online_fusion", "warp_mapping", "split_mapping", "shuffle",
                     "pointwise_fusion", "row_pipelining", "vectorize", "feature_tile"}
