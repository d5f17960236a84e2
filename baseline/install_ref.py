"""Lay the reference's ``wave_rt`` package out in baseline/_ref.

    python baseline/install_ref.py <WaveForcing checkout>

First tries the install the benchmark contract names:
    pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
                --target baseline/_ref <checkout> --no-deps
The reference builds with hatchling, which the offline wheelhouse does not
carry, so that install fails here.  The package is pure Python, so the
fallback places the checkout's ``wave_rt`` tree, unmodified, where
``pip --target`` would have put it.  baseline/_ref is git-ignored: it travels
with the working tree to the GPU boxes (where no checkout exists) and never
enters the repository's history.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
DEST = os.path.join(HERE, "_ref")


def main(src: str) -> int:
    if not os.path.isdir(os.path.join(src, "wave_rt")):
        print(f"not a WaveForcing checkout: {src}", file=sys.stderr)
        return 2
    os.makedirs(DEST, exist_ok=True)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", DEST, src, "--no-deps"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0 and os.path.isdir(os.path.join(DEST, "wave_rt")):
        print("pip install into baseline/_ref: ok")
        return 0
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["?"]
    print(f"pip install failed ({tail[0]}); placing the unmodified wave_rt package instead")
    dst = os.path.join(DEST, "wave_rt")
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    shutil.copytree(os.path.join(src, "wave_rt"), dst, ignore=shutil.ignore_patterns("__pycache__"))
    print(f"baseline/_ref/wave_rt: {sum(len(f) for _, _, f in os.walk(dst))} files")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("WF_REFERENCE", "")))
