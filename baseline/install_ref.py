"""Install the reference's quantizer modules, unmodified, under baseline/_ref.

    python baseline/install_ref.py [REFERENCE_ROOT]

The reference checkout (efsotr/test_speed_scalesweep) has no setup.py or
pyproject.toml, so ``pip install <checkout>`` refuses it.  This recipe copies
its ``bench_kernel/`` directory byte for byte into a scratch directory under
/tmp, adds packaging metadata there (and nothing else), and installs it with
the offline pip command:

    pip install --no-index --no-build-isolation --no-deps \
        --find-links /opt/wheelhouse --target baseline/_ref <scratch>

The result is ``baseline/_ref/bench_kernel/*.py``, importable as
``bench_kernel.scalesweep_mse_nvfp4_utils`` once ``baseline/_ref`` is on
sys.path.  Only bench.py (its same-box reference-kernel leg) and tests/
import it; the package never does.  ``baseline/_ref`` is git-ignored (it is
not this project's source) but travels with the working tree to a GPU host.
The copied files' SHA-256 digests are written to baseline/_ref/SOURCES.sha256
and compared against the checkout, so the install is provably unmodified.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
PYPROJECT = """\
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "test-speed-scalesweep-bench-kernel"
version = "0.0.0"

[tool.setuptools]
packages = ["bench_kernel"]
"""


def _sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def install(ref_root: str) -> None:
    src = os.path.join(ref_root, "bench_kernel")
    if not os.path.isdir(src):
        raise SystemExit(f"no bench_kernel/ under {ref_root}")
    names = sorted(n for n in os.listdir(src) if n.endswith(".py"))
    with tempfile.TemporaryDirectory(prefix="ssw_ref_") as tmp:
        pkg = os.path.join(tmp, "bench_kernel")
        os.makedirs(pkg)
        for n in names:
            shutil.copyfile(os.path.join(src, n), os.path.join(pkg, n))
        with open(os.path.join(tmp, "pyproject.toml"), "w") as f:
            f.write(PYPROJECT)
        if os.path.isdir(TARGET):
            shutil.rmtree(TARGET)
        subprocess.check_call([sys.executable, "-m", "pip", "install", "--no-index",
                               "--no-build-isolation", "--no-deps", "--find-links",
                               "/opt/wheelhouse", "--target", TARGET, tmp])
    lines = []
    for n in names:
        got = _sha(os.path.join(TARGET, "bench_kernel", n))
        want = _sha(os.path.join(src, n))
        if got != want:
            raise SystemExit(f"installed {n} differs from the checkout")
        lines.append(f"{got}  bench_kernel/{n}")
    with open(os.path.join(TARGET, "SOURCES.sha256"), "w") as f:
        f.write("\n".join(lines) + "\n")
    print(f"installed {len(names)} unmodified modules under {TARGET}")


if __name__ == "__main__":
    install(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
