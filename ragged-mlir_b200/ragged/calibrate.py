"""Refit the schedule cost model on this GPU (python -m ragged.calibrate).

Restates the reference's calibration protocol (bench/calibrate.py:1-40 of
simon-jd/ragged-mlir) for libragged_b200's schedules:

    python -m ragged.calibrate measure --output ragged/calibration/b200.json
    python -m ragged.calibrate fit ragged/calibration/b200.json --output ragged/cost_model.json
    python -m ragged.calibrate evaluate ragged/calibration/b200.json

``measure`` (needs the GPU) draws a seeded synthetic suite -- operation,
dtype, D, length distribution (the reference's five families,
bench/distributions.py:15-64), N and B -- splits it into a training group
and a held-out group, and times every schedule of every case through the
public API (CUDA events around complete calls, median of 5 after 2 warm-up
calls, L2 flushed before each call when the inputs are smaller than 4x L2).
``fit`` fits, per operation family and schedule, the six nonnegative
coefficients of ``selection.features`` that minimise the squared relative
error on the training group (NNLS on rows scaled by 1/time), picks the
margin in 0..10% that puts the most training cases within 3% of their
fastest schedule, and fits the tree chooser (``fit_chooser``) that makes
the version-4 model's choice.  ``evaluate`` reports, on the held-out group, the share of
cases whose chosen schedule is within 3% of the fastest one measured.  The
L2 capacity of the bytes-beyond-L2 term is the measuring device's.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path
import statistics
import sys

import numpy as np

from .selection import (CHOICE_FEATURES, FAMILIES, MODEL_PATH, SCHEDULES, TERMS, CostModel, TreeChooser,
                        choice_features, family, features)

DISTRIBUTIONS = ("uniform", "long_tail", "bimodal", "burst", "exponential")
WITHIN = 0.03
MARGINS = [percent / 100 for percent in range(11)]


def lengths_of(distribution: str, segments: int, total: int, rng: np.random.Generator) -> np.ndarray:
    """Seeded lengths summing to ``total`` in one of the reference's five
    families: uniform, long tail (Pareto), bimodal 90/10, a burst of 1% of
    the segments holding most rows, exponential."""
    if distribution == "uniform":
        weights = rng.uniform(0.5, 1.5, segments)
    elif distribution == "long_tail":
        weights = np.minimum(rng.pareto(1.3, segments) + 1, 1e5)
    elif distribution == "bimodal":
        weights = np.where(rng.random(segments) < 0.9, 1.0, 256.0)
    elif distribution == "exponential":
        weights = rng.exponential(1.0, segments)
    else:
        weights = np.ones(segments)
        width = max(1, segments // 100)
        start = int(rng.integers(segments - width + 1))
        weights[start:start + width] = 4096.0
    share = weights / weights.sum() * total
    lengths = np.floor(share).astype(np.int64)
    remainder = total - int(lengths.sum())
    lengths[np.argsort(-(share - lengths), kind="stable")[:remainder]] += 1
    return lengths


def suite(seed: int = 20261201, count: int = 240, max_bytes: int = 1 << 30) -> list[dict]:
    """The synthetic cases; every third one (by draw order) is held out."""
    rng = np.random.default_rng(seed)
    cases = []
    while len(cases) < count:
        op = ("sum", "max", "softmax")[int(rng.integers(3))]
        dtype = ("f32", "bf16")[int(rng.integers(2))]
        d = int((1, 2, 8, 32, 64, 128, 256, 512, 1024)[int(rng.integers(9))])
        element = 4 if dtype == "f32" else 2
        n = int(2 ** rng.uniform(12, 24))
        if n * d * element * (2 if op == "softmax" else 1) > max_bytes:
            continue
        mean_len = 2 ** rng.uniform(1, 12)
        b = max(1, min(n, int(n / mean_len)))
        distribution = DISTRIBUTIONS[int(rng.integers(len(DISTRIBUTIONS)))]
        cases.append({"id": len(cases), "op": op, "dtype": dtype, "d": d, "n": n, "b": b,
                      "distribution": distribution, "seed": int(rng.integers(1 << 30)),
                      "group": "heldout" if len(cases) % 3 == 2 else "train"})
    return cases


def measure(args: argparse.Namespace) -> None:
    import torch
    from . import ArtifactCache, Compiler, ProgramSpec
    import tempfile

    device = torch.device("cuda", 0)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    flush = torch.empty(2 * l2 // 4, dtype=torch.float32, device=device)
    cache = ArtifactCache(tempfile.mkdtemp(prefix="ragged-calibrate-"), max_specializations=4096)
    results = []
    for case in suite(args.seed, args.count):
        rng = np.random.default_rng(case["seed"])
        lengths = lengths_of(case["distribution"], case["b"], case["n"], rng)
        offsets = np.zeros(case["b"] + 1, dtype=np.int64)
        np.cumsum(lengths, out=offsets[1:])
        tdtype = torch.float32 if case["dtype"] == "f32" else torch.bfloat16
        values = torch.randn((case["n"], case["d"]), device=device, dtype=torch.float32).to(tdtype)
        dev_offsets = torch.from_numpy(offsets).to(device)
        rows = case["n"] if case["op"] == "softmax" else case["b"]
        out = torch.empty((rows, case["d"]), dtype=tdtype, device=device)
        program = Compiler().compile(ProgramSpec(case["op"], case["dtype"], case["d"], "i64"), cache)
        cold = values.numel() * values.element_size() < 4 * l2
        times = {}
        for schedule in program.schedules:
            samples = []
            for rep in range(7):
                if cold:
                    flush.add_(1)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                program.run(values, dev_offsets, out, select=schedule)
                end.record()
                torch.cuda.synchronize()
                if rep >= 2:
                    samples.append(start.elapsed_time(end) * 1000.0)
            times[schedule] = statistics.median(samples)
        results.append({**case, "max_len": int(lengths.max()), "times_us": times, "cold_l2": cold})
        print(json.dumps({k: results[-1][k] for k in ("id", "op", "dtype", "d", "n", "b", "distribution",
                                                       "times_us")}), flush=True)
    data = {"device": torch.cuda.get_device_name(device), "l2_mib": l2 / 2**20,
            "protocol": "median of 5 complete calls after 2 warm-up, CUDA events; L2 flushed when inputs < 4x L2",
            "cases": results}
    Path(args.output).parent.mkdir(parents=True, exist_ok=True)
    Path(args.output).write_text(compact_runs(data))


def compact_runs(data: dict) -> str:
    """A measurement file as JSON with one case per line."""
    head = json.dumps({k: v for k, v in data.items() if k != "cases"})[:-1]
    cases = ",\n".join(json.dumps(case, separators=(",", ":")) for case in data["cases"])
    return f'{head}, "cases": [\n{cases}\n]}}\n'



def _terms(case: dict, l2_mib: float) -> tuple[float, ...]:
    from .optimizations import Optimizations
    tile, vec = Optimizations().geometry(case["d"], case["dtype"])
    element = 4 if case["dtype"] == "f32" else 2
    return features(case["n"], case["b"], case["d"], case["max_len"], tile * vec, element, case["op"], l2_mib)


def _nnls(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    from scipy.optimize import nnls
    return nnls(a, b)[0]


def fit_coefficients(cases: list[dict], l2_mib: float) -> dict:
    """Per family and schedule: nonnegative coefficients minimising the
    squared relative error of the predicted complete-call time."""
    coefficients: dict = {}
    for fam in FAMILIES:
        chosen = [c for c in cases if family(c["op"]) == fam]
        schedules = sorted({s for c in chosen for s in c["times_us"]})
        coefficients[fam] = {}
        for schedule in schedules:
            rows = [c for c in chosen if schedule in c["times_us"]]
            a = np.array([_terms(c, l2_mib) for c in rows], dtype=np.float64)
            t = np.array([c["times_us"][schedule] for c in rows], dtype=np.float64)
            coef = _nnls(a / t[:, None], np.ones(len(rows)))
            coefficients[fam][schedule] = [round(float(x), 6) for x in coef]
    return coefficients


def _choice_row(case: dict) -> np.ndarray:
    element = 4 if case["dtype"] == "f32" else 2
    return choice_features(case["op"], case["n"], case["b"], case["d"], case["max_len"], element)


def fit_chooser(cases: list[dict], *, rounds: int = 100, leaves: int = 15, seed: int = 0) -> dict:
    """Gradient-boosted trees (scikit-learn's histogram boosting, fit time
    only) predicting each training case's fastest schedule from
    ``choice_features``, exported as the node arrays of
    ``selection.TreeChooser``.  The export is checked against scikit-learn's
    own predictions on every case, and a sample of them is recorded as
    ``checks`` that loading the model replays."""
    from sklearn.ensemble import HistGradientBoostingClassifier
    x = np.array([_choice_row(c) for c in cases])
    y = np.array([min(c["times_us"], key=c["times_us"].get) for c in cases])
    model = HistGradientBoostingClassifier(max_iter=rounds, max_leaf_nodes=leaves, learning_rate=0.1,
                                           early_stopping=False, random_state=seed)
    model.fit(x, y)
    classes = [str(c) for c in model.classes_]
    feature, threshold, left, right, value, leaf, roots, tree_class = [], [], [], [], [], [], [], []
    max_depth = 0
    for trees in model._predictors:  # one list per boosting round: a tree per class
        if len(trees) != len(classes):
            raise RuntimeError("expected one tree per class and round")
        for k, tree in enumerate(trees):
            base = len(feature)
            nodes = tree.nodes
            if np.any(nodes["is_categorical"]):  # the features are never missing, so only numeric splits matter
                raise RuntimeError("categorical splits are not exported")
            roots.append(base)
            tree_class.append(k)
            max_depth = max(max_depth, int(nodes["depth"].max()))
            for node in nodes:
                is_leaf = bool(node["is_leaf"])
                feature.append(0 if is_leaf else int(node["feature_idx"]))
                threshold.append(0.0 if is_leaf else float(node["num_threshold"]))
                left.append(base + int(node["left"]) if not is_leaf else -1)
                right.append(base + int(node["right"]) if not is_leaf else -1)
                value.append(float(node["value"]) if is_leaf else 0.0)
                leaf.append(is_leaf)
    baseline = np.asarray(model._baseline_prediction, dtype=np.float64).reshape(-1)
    if len(classes) == 2:
        raise RuntimeError("the export expects three or more schedules (one tree per class)")
    data = {"features": CHOICE_FEATURES, "classes": classes, "baseline": [float(v) for v in baseline],
            "nodes": {"feature": feature, "threshold": threshold, "left": left, "right": right, "value": value,
                      "leaf": leaf},
            "roots": roots, "tree_class": tree_class, "max_depth": max_depth}
    chooser = TreeChooser.from_dict(data)
    expected = model.predict(x)
    mine = [chooser.classes[int(np.argmax(chooser.scores(row)))] for row in x]
    if any(a != b for a, b in zip(mine, expected)):
        raise RuntimeError("exported trees disagree with scikit-learn's predictions")
    step = max(1, len(x) // 32)
    data["checks"] = [[float(v) for v in x[i]] + [str(expected[i])] for i in range(0, len(x), step)]
    return data


def within_share(model: CostModel, cases: list[dict], l2_mib: float) -> tuple[int, int, list[dict]]:
    hits, misses = 0, []
    for case in cases:
        from .optimizations import Optimizations
        tile, vec = Optimizations().geometry(case["d"], case["dtype"])
        element = 4 if case["dtype"] == "f32" else 2
        available = tuple(case["times_us"])
        chosen, _ = model.choose(case["op"], case["n"], case["b"], case["d"], case["max_len"], tile * vec, element,
                                 l2_mib=l2_mib, available=available)
        best = min(case["times_us"].values())
        if case["times_us"][chosen] <= best * (1 + WITHIN):
            hits += 1
        else:
            misses.append({"id": case["id"], "op": case["op"], "chosen": chosen,
                           "slowdown": round(case["times_us"][chosen] / best, 3)})
    return hits, len(cases), misses


def _slowdown(model: CostModel, case: dict, l2_mib: float) -> float:
    from .optimizations import Optimizations
    tile, vec = Optimizations().geometry(case["d"], case["dtype"])
    element = 4 if case["dtype"] == "f32" else 2
    chosen, _ = model.choose(case["op"], case["n"], case["b"], case["d"], case["max_len"], tile * vec, element,
                             l2_mib=l2_mib, available=tuple(case["times_us"]))
    return case["times_us"][chosen] / min(case["times_us"].values())


def fit(args: argparse.Namespace) -> None:
    data = json.loads(Path(args.runs).read_text())
    l2_mib = float(data["l2_mib"])
    train = [c for c in data["cases"] if c["group"] == "train"]
    heldout = [c for c in data["cases"] if c["group"] == "heldout"]
    coefficients = fit_coefficients(train, l2_mib)
    best_margin, best_hits = 0.0, -1
    for margin in MARGINS:
        model = CostModel(coefficients, margin, {}, l2_mib)
        hits, _, _ = within_share(model, train, l2_mib)
        if hits > best_hits:
            best_margin, best_hits = margin, hits
    linear = CostModel(coefficients, best_margin, {}, l2_mib)
    linear_held, _, _ = within_share(linear, heldout, l2_mib)
    chooser = fit_chooser(train)
    model = CostModel(coefficients, best_margin, {}, l2_mib, TreeChooser.from_dict(chooser))
    train_hits, _, _ = within_share(model, train, l2_mib)
    held_hits, held_total, held_misses = within_share(model, heldout, l2_mib)
    slowdowns = [_slowdown(model, c, l2_mib) for c in heldout]
    out = {"version": 4, "coefficients": coefficients, "margin": best_margin, "l2_mib": l2_mib, "chooser": chooser,
           "calibration": {"status": "fitted by python -m ragged.calibrate fit", "device": data["device"],
                           "runs": Path(args.runs).name, "train_cases": len(train), "heldout_cases": held_total,
                           "train_within_3pct": train_hits, "heldout_within_3pct": held_hits,
                           "heldout_share": round(held_hits / max(1, held_total), 4),
                           "heldout_geomean_slowdown": round(float(np.exp(np.mean(np.log(slowdowns)))), 4),
                           "heldout_worst_slowdown": round(max(slowdowns), 3),
                           "linear_only_heldout_share": round(linear_held / max(1, held_total), 4)}}
    # The tree arrays go on one line; the rest stays readable.
    text = json.dumps({**out, "chooser": "@chooser@"}, indent=2)
    text = text.replace('"@chooser@"', json.dumps(chooser, separators=(",", ":")))
    Path(args.output).write_text(text + "\n")
    print(json.dumps(out["calibration"]))
    for miss in held_misses:
        print("held-out miss:", json.dumps(miss))


def evaluate(args: argparse.Namespace) -> None:
    data = json.loads(Path(args.runs).read_text())
    l2_mib = float(data["l2_mib"])
    model = CostModel.load(Path(args.model))
    for group in ("train", "heldout"):
        cases = [c for c in data["cases"] if c["group"] == group]
        hits, total, _ = within_share(model, cases, l2_mib)
        print(f"{group}: {hits}/{total} within 3% of the fastest schedule ({hits / max(1, total):.1%})")


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(prog="python -m ragged.calibrate", description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(dest="command", required=True)
    m = sub.add_parser("measure")
    m.add_argument("--output", required=True)
    m.add_argument("--seed", type=int, default=20261201)
    m.add_argument("--count", type=int, default=240)
    f = sub.add_parser("fit")
    f.add_argument("runs")
    f.add_argument("--output", default=str(MODEL_PATH))
    e = sub.add_parser("evaluate")
    e.add_argument("runs")
    e.add_argument("--model", default=str(MODEL_PATH))
    args = parser.parse_args(argv)
    {"measure": measure, "fit": fit, "evaluate": evaluate}[args.command](args)


if __name__ == "__main__":
    main(sys.argv[1:])
