"""Import the upstream Cherimoya package itself.  TEST INFRASTRUCTURE ONLY.

Used by ``bench.py --impl reference`` and the ``cpu_baseline`` leg (the
upstream CPU forward timed on the host cores) and by the fixture generator
``tests/golden/make_golden.py``; never by the engine.

Where the package is looked up, first match wins:
  1. ``$CHERIMOYA_REFERENCE`` -- a source checkout (a directory holding
     ``cherimoya/``) or a pip ``--target`` directory;
  2. ``baseline/_ref`` under the repository root, a pip ``--target`` install
     of the upstream checkout (``--no-deps``: its third-party imports are
     replaced below).

The upstream package imports two third-party projects at module import time
that are not installed here: ``tangermeme`` (``predict``,
``io.extract_loci``) and ``bpnetlite`` (``logging.Logger``,
``losses.MNLLLoss``) (upstream ``cherimoya/cherimoya.py:19-20``,
``cherimoya/io.py:8``, ``cherimoya/losses.py:14``). None is on the
inference path (``cherimoya/cheri.py``, ``Cherimoya._forward_impl``,
``cherimoya/wrappers.py``, ``performance.jensen_shannon_distance``), so
stand-ins that raise when called are enough. ``cherimoya/__init__.py:14``
reads ``importlib.metadata.version('cherimoya')``; a pip install carries its
dist-info, a bare checkout gets a stand-in one.
"""

import importlib
import os
import sys
import tempfile

REPO_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PIP_TARGET = os.path.join(REPO_ROOT, "baseline", "_ref")

STUBS = {
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
}
DIST_INFO = {
    "cherimoya-0.2.1.dist-info/METADATA":
        "Metadata-Version: 2.1\nName: cherimoya\nVersion: 0.2.1\n",
}


def location():
    """Directory to put on sys.path for ``import cherimoya``, or None."""
    for root in (os.environ.get("CHERIMOYA_REFERENCE"), PIP_TARGET):
        if root and os.path.isfile(os.path.join(root, "cherimoya", "cherimoya.py")):
            return root
    return None


def available():
    return location() is not None


def import_upstream():
    """Return the upstream ``cherimoya`` package, importing it once; raises
    RuntimeError when no copy is found."""
    mod = sys.modules.get("cherimoya")
    if mod is not None and hasattr(mod, "Cherimoya"):
        return mod
    root = location()
    if root is None:
        raise RuntimeError("upstream cherimoya not found: set CHERIMOYA_REFERENCE or install "
                           "it into " + PIP_TARGET)
    os.environ.setdefault("TORCH_COMPILE_DISABLE", "1")
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    stub_dir = tempfile.mkdtemp(prefix="cherimoya_upstream_stubs_")
    files = dict(STUBS)
    has_dist = any(n.startswith("cherimoya-") and n.endswith(".dist-info")
                   for n in os.listdir(root))
    if not has_dist:
        files.update(DIST_INFO)
    for rel, text in files.items():
        path = os.path.join(stub_dir, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(text)
    sys.path.insert(0, stub_dir)
    sys.path.insert(0, root)
    importlib.invalidate_caches()
    return importlib.import_module("cherimoya")
