"""Build the REFERENCE's own CUDA extensions, unchanged, into oracle/_ref/ --
TEST INFRASTRUCTURE (the checker, never the product).

    python oracle/build_ref.py [--reference <reference tree>] [--jobs 6]

rabbit-art/CIGN JIT-compiles its kernels with torch.utils.cpp_extension
(`load` on the *_ext/ sources, `load_inline` on CUDA strings kept inside a few
Python modules).  This recipe does the same, for sm_100 (TORCH_CUDA_ARCH_LIST
10.0; the reference's default is 8.6), with the reference's own extra flags,
from the sources where they lie in the reference tree.  Nothing is copied into
the repository: every output goes to oracle/_ref/, which .gitignore lists
and which travels to the GPU box with the rest of the working tree (the
reference tree does not).

Built extensions (module name -> reference sources, loader it mirrors):

  ref_collapsed_gat      collapsed_gat_ext/collapsed_gat{.cpp,_cuda.cu}        collapsed_gat.py:19-54
  ref_gat_sideops        fused_gat_sideops_ext/fused_gat_sideops{.cpp,_cuda.cu} fused_gat_sideops.py:22-47
  ref_block_ops_d256     fused_block_ops_ext/fused_block_ops{.cpp,_cuda.cu}     fused_block_ops.py:52-74
  ref_block_ops_general  the _CPP_SOURCE/_CUDA_SOURCE strings of fused_block_ops.py:14-15
  ref_multihop_csr       multihop_csr_ext/multihop_csr_pipeline{.cpp,_cuda.cu}  multihop_csr_pipeline.py:18-35
                         (-O3 --use_fast_math, -lcusparse)
  ref_clifford_pack3     fused_clifford_pack_ext/fused_clifford_pack{.cpp,_cuda.cu}  fused_clifford_pack.py:27-45
  ref_clifford_pack_k    the _GENERIC_CPP/_GENERIC_CUDA strings of fused_clifford_pack.py:48-140
  ref_cign_pack3         generic_engine/fused_clifford_cign_pack_ext/*          generic_engine/fused_clifford_cign_pack.py:30-57
  ref_cign_pack_k        the _GENERIC_CPP/_GENERIC_CUDA strings of generic_engine/fused_clifford_cign_generic.py:18-110

The inline CUDA strings are read with `ast` (the reference modules are not
executed).  Besides the extensions, the reference's model module
generic_engine/model_cign.py is byte-compiled (py_compile) to
oracle/_ref/py/model_cign.bytecode (a .pyc under another suffix, which the
working-tree snapshot keeps), so the drop-in test can run the reference's
own, unchanged GraphCliffordNet on the GPU box over this repository's op
modules.

Each extension is built in its own process (they run in parallel), is
skipped when its .so is newer than its sources, and a failure of one does
not stop the others; the exit status is non-zero if any failed.
"""
from __future__ import annotations

import argparse
import ast
import concurrent.futures as cf
import importlib.machinery
import importlib.util
import os
import py_compile
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REFERENCE = Path("/root/reference")
ARCH = "10.0"

# name -> (kind, spec, extra_cuda_cflags, extra_ldflags)
#   kind "files":  spec = list of source paths relative to the reference root
#   kind "inline": spec = (python file, cpp variable, cuda variable)
EXTENSIONS = {
    "ref_collapsed_gat": ("files", ["collapsed_gat_ext/collapsed_gat.cpp",
                                    "collapsed_gat_ext/collapsed_gat_cuda.cu"], ["-O3"], []),
    "ref_gat_sideops": ("files", ["fused_gat_sideops_ext/fused_gat_sideops.cpp",
                                  "fused_gat_sideops_ext/fused_gat_sideops_cuda.cu"], ["-O3"], []),
    "ref_block_ops_d256": ("files", ["fused_block_ops_ext/fused_block_ops.cpp",
                                     "fused_block_ops_ext/fused_block_ops_cuda.cu"], ["-O3"], []),
    "ref_block_ops_general": ("inline", ("fused_block_ops.py", "_CPP_SOURCE", "_CUDA_SOURCE"),
                              ["-O3"], []),
    "ref_multihop_csr": ("files", ["multihop_csr_ext/multihop_csr_pipeline.cpp",
                                   "multihop_csr_ext/multihop_csr_pipeline_cuda.cu"],
                         ["-O3", "--use_fast_math"], ["-lcusparse"]),
    "ref_clifford_pack3": ("files", ["fused_clifford_pack_ext/fused_clifford_pack.cpp",
                                     "fused_clifford_pack_ext/fused_clifford_pack_cuda.cu"],
                           ["-O3"], []),
    "ref_clifford_pack_k": ("inline", ("fused_clifford_pack.py", "_GENERIC_CPP", "_GENERIC_CUDA"),
                            ["-O3"], []),
    "ref_cign_pack3": ("files", [
        "generic_engine/fused_clifford_cign_pack_ext/fused_clifford_switch_pack.cpp",
        "generic_engine/fused_clifford_cign_pack_ext/fused_clifford_switch_pack_cuda.cu"],
        ["-O3"], []),
    "ref_cign_pack_k": ("inline", ("generic_engine/fused_clifford_cign_generic.py",
                                   "_GENERIC_CPP", "_GENERIC_CUDA"), ["-O3"], []),
}

PY_MODULES = {"model_cign": "generic_engine/model_cign.py"}


def reference_root():
    """The reference tree (CIGN_REFERENCE_ROOT, else the default location), or
    None where it is absent (e.g. on the GPU box)."""
    ref = Path(os.environ.get("CIGN_REFERENCE_ROOT", str(DEFAULT_REFERENCE)))
    return ref if ref.is_dir() else None


def so_path(name: str) -> Path:
    return OUT / name / f"{name}.so"


def load_extension(name: str):
    """Import a built reference extension from oracle/_ref/ (torch must be
    imported first; used by tests and the golden script on the GPU box)."""
    import torch  # noqa: F401  (the extension links against torch's libraries)
    path = so_path(name)
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run oracle/build_ref.py where the "
                                "reference tree is present)")
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _inline_strings(pyfile: Path, cpp_var: str, cuda_var: str):
    tree = ast.parse(pyfile.read_text())
    found = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 \
                and isinstance(node.targets[0], ast.Name) and node.targets[0].id in (cpp_var, cuda_var):
            found[node.targets[0].id] = ast.literal_eval(node.value)
    missing = {cpp_var, cuda_var} - set(found)
    if missing:
        raise RuntimeError(f"{pyfile}: no string constant {sorted(missing)}")
    return found[cpp_var], found[cuda_var]


def _sources(ref: Path, name: str):
    kind, spec, _, _ = EXTENSIONS[name]
    if kind == "files":
        return [ref / s for s in spec]
    return [ref / spec[0]]


def _up_to_date(ref: Path, name: str) -> bool:
    so = so_path(name)
    if not so.exists():
        return False
    t = so.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in _sources(ref, name)) and \
        Path(__file__).stat().st_mtime <= t


def build_one(ref: Path, name: str, verbose: bool = False) -> Path:
    """Build one extension in this process (called in a child process)."""
    os.environ["TORCH_CUDA_ARCH_LIST"] = ARCH
    from torch.utils import cpp_extension as ce
    kind, spec, cuda_flags, ldflags = EXTENSIONS[name]
    bdir = OUT / name
    bdir.mkdir(parents=True, exist_ok=True)
    common = dict(name=name, extra_cflags=["-O3"], extra_cuda_cflags=list(cuda_flags),
                  extra_ldflags=list(ldflags), build_directory=str(bdir), verbose=verbose)
    if kind == "files":
        ce.load(sources=[str(ref / s) for s in spec], **common)
    else:
        cpp, cuda = _inline_strings(ref / spec[0], spec[1], spec[2])
        ce.load_inline(cpp_sources=cpp, cuda_sources=cuda, functions=None, with_cuda=True, **common)
    if not so_path(name).exists():
        raise RuntimeError(f"{name}: build finished without {so_path(name)}")
    for obj in bdir.glob("*.o"):  # intermediates: only the .so travels
        obj.unlink()
    so_path(name).touch()
    return so_path(name)


def compile_py(ref: Path) -> list:
    out = []
    pydir = OUT / "py"
    pydir.mkdir(parents=True, exist_ok=True)
    for mod, rel in PY_MODULES.items():
        dst = pydir / f"{mod}.bytecode"
        py_compile.compile(str(ref / rel), cfile=str(dst), dfile=rel, doraise=True)
        out.append(dst)
    return out


def build_all(ref: Path = DEFAULT_REFERENCE, jobs: int = 6, names=None, verbose: bool = False):
    """Build every (or the named) reference extension; returns {name: error or None}."""
    ref = Path(ref)
    if not ref.is_dir():
        raise FileNotFoundError(f"reference tree not found at {ref}")
    OUT.mkdir(parents=True, exist_ok=True)
    names = list(names or EXTENSIONS)
    results = {}
    todo = [n for n in names if not _up_to_date(ref, n)]
    for n in names:
        if n not in todo:
            results[n] = None
    env = dict(os.environ, TORCH_CUDA_ARCH_LIST=ARCH, MAX_JOBS="2")

    def run(n):
        cmd = [sys.executable, str(Path(__file__).resolve()), "--reference", str(ref), "--one", n]
        res = subprocess.run(cmd, capture_output=True, text=True, env=env)
        return n, (None if res.returncode == 0 else (res.stdout + res.stderr)[-4000:])

    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for n, err in ex.map(run, todo):
            results[n] = err
    compile_py(ref)
    return results


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--reference", default=str(DEFAULT_REFERENCE))
    ap.add_argument("--jobs", type=int, default=6)
    ap.add_argument("--one", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("names", nargs="*")
    args = ap.parse_args(argv)
    if args.one:
        build_one(Path(args.reference), args.one, args.verbose)
        return 0
    results = build_all(Path(args.reference), args.jobs, args.names or None, args.verbose)
    bad = {n: e for n, e in results.items() if e}
    for n in results:
        print(f"{n}: {'FAILED' if n in bad else 'ok'} ({so_path(n)})")
    for n, e in bad.items():
        print(f"---- {n}\n{e}")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
