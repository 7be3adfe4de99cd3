"""Install the unmodified reference package into baseline/_ref (git-ignored).

    python baseline/install_ref.py --reference <checkout of kani-tts-2-openai-server>

(or set KANI_REFERENCE_DIR).  The reference checkout has neither setup.py nor
pyproject.toml, so ``pip install --target baseline/_ref <checkout>`` refuses it
("Directory ... is not installable").  The package is therefore installed the
way pip would lay out a pure-Python package: the ``kani_tts`` directory's
``.py`` files are copied byte for byte into ``baseline/_ref/kani_tts``.  The
copies are never edited; ``baseline/_ref/MANIFEST.json`` records each file's
SHA-256 next to the source's, and ``baseline/reference.py`` checks them
before importing.

baseline/_ref is git-ignored (it is the reference's code, not this
project's), and it travels with the working tree to the GPU host, where the
reference checkout itself does not exist.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def try_pip(reference: Path) -> str:
    """The installation the benchmark contract names; its outcome is recorded."""
    scratch = Path("/tmp") / "kani_ref_pip_probe"
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
           "--find-links", "/opt/wheelhouse", "--target", str(scratch), str(reference)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    except (OSError, subprocess.TimeoutExpired) as exc:
        return f"pip did not run: {exc}"
    lines = [ln for ln in (r.stdout + r.stderr).splitlines() if ln.strip()]
    shutil.rmtree(scratch, ignore_errors=True)
    return f"rc={r.returncode}: " + (lines[-1] if lines else "")


def install(reference: Path) -> dict:
    src = reference / "kani_tts"
    if not (src / "optimized_decode.py").exists():
        raise SystemExit(f"{src} does not hold the kani_tts package")
    pip_outcome = try_pip(reference)
    dst = TARGET / "kani_tts"
    if dst.exists():
        shutil.rmtree(dst)
    dst.mkdir(parents=True)
    files = {}
    for f in sorted(src.glob("*.py")):
        shutil.copyfile(f, dst / f.name)
        h = sha256(dst / f.name)
        if h != sha256(f):
            raise SystemExit(f"copy of {f.name} differs from its source")
        files[f.name] = h
    manifest = {"package": "kani_tts", "files": files, "pip_install_outcome": pip_outcome,
                "method": "byte-for-byte copy of the package's .py files (pip refuses the checkout)"}
    (TARGET / "MANIFEST.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return manifest


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=os.environ.get("KANI_REFERENCE_DIR"),
                    help="path of the reference checkout (or set KANI_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set KANI_REFERENCE_DIR")
    m = install(Path(args.reference))
    print(f"installed {len(m['files'])} files into {TARGET / 'kani_tts'}; pip: {m['pip_install_outcome']}")


if __name__ == "__main__":
    main()
