"""Build the reference's own CUDA extension into ``oracle/_ref/`` -- TEST AND
BASELINE INFRASTRUCTURE ONLY.

    python -m oracle.build_ref [--force]

Compiles the reference's three extension sources
(``aq_kernels/aq_lut.cu``, ``aq_kernels/aq_lut_gqa.cu``,
``aq_kernels/fused_linear_encode.cu``) unchanged, where they lie in the
reference checkout, with the nvcc flags of the reference's ``setup.py``
(``-O3``, plus ``--use_fast_math`` for all but ``aq_lut``) and the sm_100a
target, through ``torch.utils.cpp_extension`` (the reference is a torch
extension: its sources include the torch headers and bind with pybind11).
Only the built modules land here, under ``oracle/_ref/<name>/<name>.so``;
no reference source is copied.  The modules travel with the repository to
a GPU host (they link against the torch libraries of the same image), where
``load(name)`` imports them without the reference checkout.

They serve two purposes, both outside the product: GPU tests compare this
package's fp16 ``aq_kernels`` drop-ins with the reference kernels on the same
inputs, and ``bench.py``'s reference arm times the reference's CUDA decode
chain beside its CPU one.  ``laprune_b200`` never imports anything here.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAMES = ("aq_lut", "aq_lut_gqa", "fused_linear_encode")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def reference_root() -> Path:
    return Path(os.environ.get("LAPRUNE_REFERENCE", "/root/reference"))


def module_path(name: str) -> Path:
    return OUT / name / f"{name}.so"


def available(name: str = "aq_lut_gqa") -> bool:
    return module_path(name).exists()


def build(force: bool = False, verbose: bool = False) -> list[Path]:
    """Compile every reference extension whose source is present (no-op for
    modules already built, unless ``force``).  Returns the built paths."""
    src_dir = reference_root() / "aq_kernels"
    if not src_dir.is_dir():
        return [module_path(n) for n in NAMES if module_path(n).exists()]
    from torch.utils import cpp_extension
    built = []
    for name in NAMES:
        src = src_dir / f"{name}.cu"
        so = module_path(name)
        if so.exists() and not force and so.stat().st_mtime >= src.stat().st_mtime:
            built.append(so)
            continue
        bdir = OUT / name
        bdir.mkdir(parents=True, exist_ok=True)
        flags = ["-O3"] if name == "aq_lut" else ["-O3", "--use_fast_math"]
        cpp_extension.load(name=name, sources=[str(src)], extra_cuda_cflags=flags + ARCH,
                           build_directory=str(bdir), verbose=verbose, with_cuda=True,
                           is_python_module=True)
        # keep only the module: the object files and ninja state stay out of
        # the snapshot that travels to the GPU host
        for p in bdir.iterdir():
            if p.name != so.name:
                if p.is_file():
                    p.unlink()
        built.append(so)
    return built


_mods: dict = {}


def load(name: str):
    """Import one built reference module (raises ImportError if absent)."""
    mod = _mods.get(name)
    if mod is None:
        so = module_path(name)
        if not so.exists():
            raise ImportError(f"reference extension {name} not built (python -m oracle.build_ref)")
        import torch  # noqa: F401  (the module links against torch's libraries)
        spec = importlib.util.spec_from_file_location(name, so)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _mods[name] = mod
    return mod


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    for p in build(force=args.force, verbose=args.verbose):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
