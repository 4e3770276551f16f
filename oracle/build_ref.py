"""TEST INFRASTRUCTURE — compile the reference's own AVX2 BSR kernel.

Builds ``ssalaad/cpu_sparse/bsr_addmm_avx2.cpp`` of the S-SALAAD sources,
where they lie (read-only, never copied), into ``oracle/_ref/`` as a Python
extension module named ``slr_ref_avx2``.  The reference loads the same file
with ``torch.utils.cpp_extension.load`` and the flags ``-O3 -mavx2 -mfma``
(ssalaad/cpu_sparse/bsr_addmm_avx2.py:25-39); this recipe calls g++ directly
with those flags plus torch's include and library paths, so nothing of the
reference's build machinery runs.

The module is the timed CPU baseline (``cpu_baseline.kind = "reference"``) and
a second pin for the C oracle.  It is built here, where the reference sources
exist, and travels to the GPU box as a prebuilt ``.so``; it is listed in
.gitignore so it never enters the history.

The reference project's root directory comes from the caller: the ``root``
argument of :func:`build`, the ``--ref-root`` option, or the environment
variable ``SLR_REFERENCE_ROOT``.  Without any of them nothing is built and a
prebuilt module, if present, is used as is.

Usage:  python oracle/build_ref.py --ref-root DIR [--force]
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "slr_ref_avx2"
SRC_IN_PROJECT = Path("ssalaad/cpu_sparse/bsr_addmm_avx2.cpp")  # path within the reference project


def output_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return OUT_DIR / f"{MODULE}{suffix}"


def build(root: Path | str | None = None, force: bool = False, quiet: bool = False) -> Path | None:
    """Compile the reference kernel of the reference project at `root`
    (default: $SLR_REFERENCE_ROOT); returns the module path, or None when the
    reference sources are absent (as on the GPU box, which uses the prebuilt
    file)."""
    out = output_path()
    stamp = OUT_DIR / "source.sha1"
    root = root if root is not None else os.environ.get("SLR_REFERENCE_ROOT")
    src = Path(root) / SRC_IN_PROJECT if root else None
    if src is None or not src.is_file():
        return out if out.is_file() else None
    digest = hashlib.sha1(src.read_bytes()).hexdigest()
    if out.is_file() and stamp.is_file() and stamp.read_text().strip() == digest and not force:
        return out
    import torch
    from torch.utils import cpp_extension

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    cmd = ["g++", "-O3", "-mavx2", "-mfma", "-shared", "-fPIC", "-std=c++17",
           f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-fopenmp"]
    for inc in cpp_extension.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-isystem", sysconfig.get_paths()["include"], str(src), "-o", str(out),
            f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
            f"-Wl,-rpath,{torch_lib}"]
    if not quiet:
        print("[oracle/build_ref]", " ".join(cmd[:6]), "...", file=sys.stderr)
    subprocess.run(cmd, check=True)
    stamp.write_text(digest + "\n")
    return out


def load():
    """Import the prebuilt reference module (requires ``import torch`` first)."""
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    path = output_path()
    if not path.is_file():
        raise FileNotFoundError(f"reference AVX2 kernel not built: {path}")
    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", type=Path, default=None,
                    help="root of the S-SALAAD reference project (default: $SLR_REFERENCE_ROOT)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    p = build(a.ref_root, a.force)
    print(p if p else "reference sources absent; nothing built")
    sys.exit(0 if p else 1)
