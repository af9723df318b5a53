"""Shared pytest setup: the `gpu` marker and the package path.

Tests marked `gpu` need an sm_100 GPU and the built libwamb.so; everything
else runs on CPU. The importable package (`wam_ops`) lives under
`wam-egale_b200/`, which is put on sys.path here.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "wam-egale_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libwamb.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.fail(f"gpu tests need sm_100 (B200); got sm_{major}{minor}")
    return torch.device("cuda", 0)


def parity_markdown(rows):
    """The recorded parity results as a markdown table."""
    out = ["| case | output | cos | max abs err | allowance at the max | E_ref (reference in bf16) |",
           "|---|---|---|---|---|---|"]
    for r in rows:
        if "vs_unquantized" in r:
            extra = f"vs fp8 model; vs fp32: cos {r['vs_unquantized']['cos']:.6f}, max {r['vs_unquantized']['max_abs']:.4f}"
            out.append(f"| {r['name']} | fp8 | {r['cos']:.7f} | {r['max_abs']:.5f} | {extra} | |")
            continue
        e = f"{r['E_ref']:.4f}" if "E_ref" in r else ""
        out.append(f"| {r['name']} | {r['dtype']} | {r['cos']:.7f} | {r['max_abs']:.5f} | "
                   f"{r['bound_at_max']:.5f} | {e} |")
    return "\n".join(out) + "\n"


def pytest_sessionfinish(session, exitstatus):
    """Write the parity results the tests recorded (blockutil.RESULTS) to
    the file named by WAMB_PARITY_OUT, if set: JSON, or a markdown table
    when the name ends in .md."""
    import json
    import os
    path = os.environ.get("WAMB_PARITY_OUT")
    if not path:
        return
    mod = sys.modules.get("blockutil")
    rows = list(getattr(mod, "RESULTS", []))
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    text = parity_markdown(rows) if path.endswith(".md") else json.dumps(rows, indent=1) + "\n"
    Path(path).write_text(text)
