"""Install the reference into ``baseline/_ref`` (git-ignored; it travels to the GPU box with the working tree).

    python tests/install_reference.py <checkout of the reference>      (or HOLMES_REFERENCE=<checkout>)

* its ``llama3fhe`` package, unchanged, by ``pip install --no-index --no-build-isolation --no-deps --target`` from a
  temporary copy (the build writes into its source tree; ``--no-deps`` because the reference pins ``triton==3.3.1``,
  which the wheelhouse does not have and which the engine's CUDA packers replace);
* its ``tests/`` and ``assets/`` directories, copied beside it, so that ``tests/easyfhe_shim_plugin.py`` can run the
  reference's own test files on this engine (``tests/test_gpu_reference_suite.py``).

Nothing here is imported by the product; the reference's EasyFHE engine itself is not part of the reference and is
not installed (this engine stands in for it).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TARGET = os.path.join(ROOT, "baseline", "_ref")


def main(reference: str) -> None:
    if not os.path.isfile(os.path.join(reference, "pyproject.toml")):
        raise SystemExit(f"{reference} is not a checkout of the reference")
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "src")
        shutil.copytree(reference, src, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
                        "/opt/wheelhouse", "--no-deps", "--upgrade", "--target", TARGET, src], check=True)
    for sub in ("tests", "assets"):
        dst = os.path.join(TARGET, sub)
        if os.path.isdir(dst):
            shutil.rmtree(dst)
        shutil.copytree(os.path.join(reference, sub), dst, ignore=shutil.ignore_patterns("__pycache__"))
    print(f"reference installed in {TARGET}")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HOLMES_REFERENCE", "")
    if not ref:
        raise SystemExit("usage: python tests/install_reference.py <checkout of the reference>")
    main(ref)
