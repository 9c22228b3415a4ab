import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "rust-llm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


# Parity counters of the -m gpu tests, per workload: rows compared, tokens
# equal, boundary cases (the oracle's draw or cutoff within 1e-6 of a CDF
# boundary, where the token may differ), kept-set checks. Written as JSON to
# $RL_PARITY_OUT at the end of the session when that variable is set.
PARITY = {}


def parity_add(key, **counts):
    d = PARITY.setdefault(key, {})
    for k, v in counts.items():
        d[k] = d.get(k, 0) + int(v)


def pytest_sessionfinish(session, exitstatus):
    out = os.environ.get("RL_PARITY_OUT")
    if out and PARITY:
        with open(out, "w") as f:
            json.dump({"exitstatus": int(exitstatus), "workloads": PARITY}, f, indent=1, sort_keys=True)
