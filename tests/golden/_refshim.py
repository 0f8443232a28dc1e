"""Import the upstream Cherimoya package (read-only checkout) for fixture generation.

The upstream package imports two third-party projects at module import time
that are not installed in this environment: ``tangermeme`` (``predict`` and
``io.extract_loci``) and ``bpnetlite`` (``logging.Logger`` and
``losses.MNLLLoss``). None of them is on the inference hot path
(``cherimoya/cheri.py``, ``Cherimoya._forward_impl``, ``wrappers.py``,
``performance.jensen_shannon_distance``), so minimal stand-ins that raise
if called are enough to import it. ``cherimoya/__init__.py:14`` also calls
``importlib.metadata.version('cherimoya')``, so a fake dist-info is added.

This module is used only by ``make_golden.py`` on a machine that has the
upstream checkout; nothing under ``tests/`` that runs in CI imports it.
"""

import importlib
import os
import sys
import tempfile

REFERENCE_ROOT = os.environ.get("CHERIMOYA_REFERENCE", "/root/reference")

_STUBS = {
    "tangermeme/__init__.py": "",
    "tangermeme/io.py": (
        "def extract_loci(*args, **kwargs):\n"
        "    raise RuntimeError('tangermeme stand-in: extract_loci unavailable')\n"),
    "tangermeme/predict.py": (
        "def predict(*args, **kwargs):\n"
        "    raise RuntimeError('tangermeme stand-in: predict unavailable')\n"),
    "bpnetlite/__init__.py": "",
    "bpnetlite/logging.py": (
        "class Logger:\n"
        "    def __init__(self, *args, **kwargs):\n"
        "        pass\n"
        "    def add(self, *args, **kwargs):\n"
        "        pass\n"
        "    def save(self, *args, **kwargs):\n"
        "        pass\n"),
    "bpnetlite/losses.py": (
        "def MNLLLoss(*args, **kwargs):\n"
        "    raise RuntimeError('bpnetlite stand-in: MNLLLoss unavailable')\n"),
    "cherimoya-0.2.1.dist-info/METADATA": (
        "Metadata-Version: 2.1\nName: cherimoya\nVersion: 0.2.1\n"),
}


def import_reference():
    """Return the upstream ``cherimoya`` package, importing it once."""
    if "cherimoya" in sys.modules and hasattr(sys.modules["cherimoya"], "Cherimoya"):
        return sys.modules["cherimoya"]
    if not os.path.isdir(os.path.join(REFERENCE_ROOT, "cherimoya")):
        raise RuntimeError("upstream checkout not found at " + REFERENCE_ROOT)
    os.environ.setdefault("TORCH_COMPILE_DISABLE", "1")
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    stub_dir = tempfile.mkdtemp(prefix="cherimoya_refshim_")
    for rel, text in _STUBS.items():
        path = os.path.join(stub_dir, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(text)
    sys.path.insert(0, stub_dir)
    sys.path.insert(0, REFERENCE_ROOT)
    importlib.invalidate_caches()
    return importlib.import_module("cherimoya")
