"""Shared pytest setup: the `gpu` marker, import paths and the built libraries.

Tests marked `gpu` run the sm_100a kernels through the C ABI and compare them
with the CPU oracle (oracle/, a restatement of the reference CPU backend).
Everything else runs on a CPU-only machine.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "random-things_b200", REPO / "oracle", REPO / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import xn_oracle

    xn_oracle.build()
    return xn_oracle


@pytest.fixture(scope="session")
def xn():
    """The product binding; on a GPU run the library must be present and loadable."""
    import xn_fused

    xn_fused.lib()
    return xn_fused


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")


def pytest_terminal_summary(terminalreporter):
    """Per-op parity summary of every assert_close check of the session: the
    largest per-element relative error (f32) and the ulp histogram (bf16 /
    f16). With XN_PARITY_LOG set, the records are also written there as JSON."""
    helpers = sys.modules.get("helpers")
    recs = getattr(helpers, "RECORDS", None) if helpers is not None else None
    if not recs:
        return
    import json
    import os

    agg: dict = {}
    for r in recs:
        key = (r["what"].split(" ")[0], r["dtype"])
        a = agg.setdefault(key, {"checks": 0, "elements": 0, "max_rel": 0.0, "max_rel_raw": 0.0,
                                 "ulp": {"0": 0, "1": 0, ">1 (within allowance)": 0}})
        a["checks"] += 1
        a["elements"] += r["n"]
        if "max_rel" in r:
            a["max_rel"] = max(a["max_rel"], r["max_rel"])
            a["max_rel_raw"] = max(a["max_rel_raw"], r.get("max_rel_raw", r["max_rel"]))
        for k, v in r.get("ulp_hist", {}).items():
            a["ulp"][k] += v
    tr = terminalreporter
    tr.section("parity summary (per element, against the oracle)")
    for (op, dt), a in sorted(agg.items()):
        if dt == "f32":
            tr.write_line(f"{op:<22} {dt:<5} checks {a['checks']:>4}  elements {a['elements']:>12}  "
                          f"max rel err {a['max_rel']:.2e} (before allowance {a['max_rel_raw']:.2e})")
        else:
            u = a["ulp"]
            tr.write_line(f"{op:<22} {dt:<5} checks {a['checks']:>4}  elements {a['elements']:>12}  "
                          f"ulp 0: {u['0']}  1: {u['1']}  >1 within allowance: {u['>1 (within allowance)']}")
    path = os.environ.get("XN_PARITY_LOG")
    if path:
        with open(path, "w") as fh:
            json.dump({"records": recs, "per_op": {f"{k[0]} {k[1]}": v for k, v in agg.items()}}, fh)
