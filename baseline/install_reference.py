"""Install the unmodified reference (tusharsonthalia/diffusion-llm) into baseline/_ref.

    python baseline/install_reference.py --src PATH_TO_REFERENCE_CHECKOUT

The reference's pyproject.toml declares no build backend and no package list, so setuptools'
flat-layout discovery refuses it (several top-level packages), it asks for Python >= 3.13
(this image has 3.12) and its dependencies include modal and torch >= 2.14.1, which are not
installable offline. The recipe therefore copies the checkout to a temporary directory,
appends a package list to the copy's pyproject.toml (model, kernels, bench, sample,
inference, train as namespace packages; infra and scripts are the Modal harness and data
preparation) and runs

    pip install --no-index --no-build-isolation --no-deps --ignore-requires-python
                --find-links /opt/wheelhouse --target baseline/_ref <copy>

The installed Python sources are byte-identical to the reference's (checked after the
install). baseline/_ref is git-ignored; it travels with the working tree to the GPU box,
where the tests of the reference's own callers and the Triton comparison import it.
"""

from __future__ import annotations

import argparse
import filecmp
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
PACKAGES = ("model", "kernels", "bench", "sample", "inference", "train")

PACKAGE_LIST = """
[tool.setuptools.packages.find]
include = [{names}]
namespaces = true
"""


def install(src: str) -> list[str]:
    with tempfile.TemporaryDirectory() as tmp:
        copy = os.path.join(tmp, "reference")
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        for root, dirs, files in os.walk(copy):
            for name in dirs + files:
                os.chmod(os.path.join(root, name), 0o755 if name in dirs else 0o644)
        names = ", ".join(f'"{p}", "{p}.*"' for p in PACKAGES)
        with open(os.path.join(copy, "pyproject.toml"), "a") as f:
            f.write(PACKAGE_LIST.format(names=names))
        if os.path.exists(TARGET):
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--no-deps", "--ignore-requires-python", "--find-links", "/opt/wheelhouse",
               "--target", TARGET, copy]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"pip install failed:\n{r.stdout}\n{r.stderr}")
    # every installed module is the reference's file, unchanged
    checked = []
    for pkg in PACKAGES:
        for name in sorted(os.listdir(os.path.join(src, pkg))):
            if not name.endswith(".py"):
                continue
            a, b = os.path.join(src, pkg, name), os.path.join(TARGET, pkg, name)
            if not filecmp.cmp(a, b, shallow=False):
                raise RuntimeError(f"{b} differs from {a}")
            checked.append(f"{pkg}/{name}")
    return checked


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True, help="a checkout of the reference")
    files = install(ap.parse_args().src)
    print(f"installed {len(files)} modules into {TARGET}: {' '.join(files)}")
