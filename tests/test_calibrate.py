"""Cost-model calibration on CPU: the fit recovers generating coefficients
and the chosen schedules follow them (as the reference's
test/python/test_calibrate.py checks its fit)."""
from __future__ import annotations

import numpy as np

from ragged import calibrate
from ragged.selection import CostModel, family


def synthetic_runs(coefficients, l2_mib=126.0):
    cases = []
    for case in calibrate.suite(seed=7, count=90):
        case = dict(case, max_len=max(1, case["n"] // max(1, case["b"]) * 3))
        times = {}
        fam = family(case["op"])
        for schedule, coef in coefficients[fam].items():
            terms = calibrate._terms(case, l2_mib)
            times[schedule] = float(np.dot(coef, terms))
        cases.append(dict(case, times_us=times))
    return cases


def test_fit_recovers_generating_coefficients():
    truth = {"reduce": {"classified": [12.0, 0.2, 0.0, 0.05, 0.0, 0.0],
                        "naive": [6.0, 0.22, 3.0, 0.3, 0.0, 0.0],
                        "rowbalanced": [10.0, 0.17, 0.0, 0.02, 0.0, 0.0]},
             "softmax": {"classified": [14.0, 0.4, 0.5, 0.05, 0.0, 0.0],
                         "naive": [6.0, 0.5, 6.0, 0.3, 0.0, 0.0]}}
    cases = synthetic_runs(truth)
    fitted = calibrate.fit_coefficients(cases, 126.0)
    for fam, schedules in truth.items():
        for schedule, coef in schedules.items():
            np.testing.assert_allclose(fitted[fam][schedule], coef, rtol=1e-3, atol=1e-3)
    model = CostModel(fitted, 0.0, {}, 126.0)
    hits, total, misses = calibrate.within_share(model, cases, 126.0)
    assert hits == total, misses


def test_suite_is_seeded_and_split():
    a, b = calibrate.suite(seed=3, count=30), calibrate.suite(seed=3, count=30)
    assert a == b
    assert {c["group"] for c in a} == {"train", "heldout"}
    for distribution in calibrate.DISTRIBUTIONS:
        lengths = calibrate.lengths_of(distribution, 100, 10_000, np.random.default_rng(1))
        assert lengths.sum() == 10_000 and (lengths >= 0).all()


def test_tree_chooser_fit_reproduces_its_labels():
    """A fastest schedule that depends on N and D only: the exported trees
    agree with scikit-learn (fit_chooser raises otherwise), replay their
    recorded checks on load, and choose the fastest schedule on held-out
    cases of the same rule."""
    from ragged.selection import TreeChooser

    def runs(seed, count):
        cases = []
        for case in calibrate.suite(seed=seed, count=count):
            case = dict(case, max_len=max(1, case["n"] // max(1, case["b"]) * 3))
            small, wide = case["n"] < 2**16, case["d"] >= 256
            best = "naive" if small else ("classified" if wide else "rowbalanced")
            case["times_us"] = {s: (10.0 if s == best else 20.0) for s in ("classified", "naive", "rowbalanced")}
            cases.append(case)
        return cases

    train, heldout = runs(11, 400), runs(12, 120)
    data = calibrate.fit_chooser(train, rounds=30)
    chooser = TreeChooser.from_dict(data)
    assert data["checks"] and chooser.max_depth >= 1
    fitted = calibrate.fit_coefficients(train, 126.0)
    model = CostModel(fitted, 0.0, {}, 126.0, chooser)
    hits, total, misses = calibrate.within_share(model, heldout, 126.0)
    assert hits >= 0.95 * total, misses


def test_shipped_model_reproduces_its_recorded_held_out_share():
    """The shipped cost model, evaluated on the shipped B200 measurements,
    gives exactly the held-out share its calibration entry records (and
    that share is at least 90 %)."""
    import json
    from pathlib import Path
    from ragged import selection
    model = selection.default_model()
    data = json.loads((Path(selection.__file__).parent / "calibration" / "b200.json").read_text())
    heldout = [c for c in data["cases"] if c["group"] == "heldout"]
    hits, total, _ = calibrate.within_share(model, heldout, float(data["l2_mib"]))
    assert total == model.calibration["heldout_cases"]
    assert hits == model.calibration["heldout_within_3pct"]
    assert hits >= 0.9 * total


def test_measurement_files_are_one_case_per_line():
    import json
    data = {"device": "x", "l2_mib": 1.0, "protocol": "p",
            "cases": [{"id": 0, "times_us": {"naive": 1.5}}, {"id": 1, "times_us": {"naive": 2.0}}]}
    text = calibrate.compact_runs(data)
    assert json.loads(text) == data
    assert len(text.strip().splitlines()) == 4
