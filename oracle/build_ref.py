"""Build the reference's own CUDA kernel as a comparison oracle (test
infrastructure only).

Compiles cuda/binding.cpp and cuda/paged_attention.cu FROM THE REFERENCE
CHECKOUT (read in place, never copied into this repository) into a torch
extension module at oracle/_ref/ref_paged_attention*.so, for sm_100 (the
reference passes no arch flags; worker/llama.py:82-84 JIT-builds with -O3 for
the build host's GPU). oracle/_ref/ is git-ignored; the built .so travels to
the GPU box with the working tree, where tests and the bench load it with
load_ref_module() to check parity against and time the reference kernel.

    python oracle/build_ref.py [/path/to/reference]

Without an argument the checkout is found by oracle/refroot.py
(PDB_REFERENCE_ROOT, else a ``reference`` directory beside this repository).
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "ref_paged_attention"


def built_path() -> Path | None:
    hits = sorted(OUT.glob(f"{NAME}*.so"))
    return hits[0] if hits else None


def build(ref_root: Path | None = None, verbose: bool = False) -> Path | None:
    if ref_root is None:
        from oracle.refroot import reference_root
        ref_root = reference_root()
    if ref_root is None:
        return built_path()
    src = [ref_root / "cuda" / "binding.cpp", ref_root / "cuda" / "paged_attention.cu"]
    if not all(p.exists() for p in src):
        return built_path()
    have = built_path()
    if have is not None and all(p.stat().st_mtime <= have.stat().st_mtime for p in src):
        return have
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load
    OUT.mkdir(parents=True, exist_ok=True)
    load(name=NAME, sources=[str(p) for p in src], extra_cuda_cflags=["-O3"],
         extra_cflags=["-O3"], build_directory=str(OUT), verbose=verbose)
    return built_path()


def load_ref_module():
    """Import the prebuilt reference extension (None if it was not built)."""
    path = built_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against libtorch)
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(path))
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    sys.path.insert(0, str(HERE.parent))
    print(build(Path(sys.argv[1]) if len(sys.argv) > 1 else None, verbose=True))
