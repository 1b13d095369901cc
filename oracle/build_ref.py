"""Build recipe for the reference's own CUDA kernel on the B200 — TEST INFRASTRUCTURE.

The reference operator (kernels/moe_w4a16_h200/moe_w4a16.py, "moe.py" below) compiles its one persistent kernel
``moe_fused`` at run time: ``_ext(defines)`` (moe.py:3081-3106) hands ``CUDA_SRC`` to the module's own
``load_inline`` override (moe.py:3866-3883), which rewrites the source per build (GF(2) decoder, handoff, M=1
program) and calls ``torch.utils.cpp_extension.load_inline``.  This script drives that stock path from the
reference checkout, unmodified, in a container without a GPU, and keeps only the built extension modules:

* the device is the B200 (compute capability 10.0); ``_ext`` derives its ``-gencode`` flag from it
  (moe.py:3091-3092), so ``torch.cuda.get_device_capability`` is answered with (10, 0) while the builds run;
* the builds are the variants ``kernel_fn`` picks by token count M (moe.py:3384-3393, :3956-3969), with the
  reference's PRMT scale decode (``-DOKC_PRMTSC=1``, chosen by prepare() for weights whose scale bytes are
  positive normals, moe.py:3337-3338): TINY (M <= 4), TINY2 (M <= 8), MID (M <= 16), the M = 1 program build,
  and for M >= 17 **MAIN_FALLBACK_DEFINES in place of the WGS MAIN build**: WGS issues ``wgmma``, which does not
  exist on sm_100, and the reference itself falls back to this build when WGS cannot run (``_main_defines``,
  moe.py:3277-3282);
* each build gets the reference's own admission routine (``ADMISSION``, the moe.py string that WGS builds
  already carry) appended as ``xc_admission``, so the caller can check with cudaOccupancyMaxActiveBlocksPerMultiprocessor
  that one CTA per SM fits before a launch (the kernel's grid barrier, moe.py:2617-2641, needs every CTA resident).

Outputs go to ``oracle/_ref/`` only: one ``.so`` per build and ``manifest.json`` (build name -> module name, file,
defines).  The intermediate sources stay in a temporary directory and are deleted; nothing of the reference's
source enters this repository.  ``oracle/okc_ref.py`` loads the modules on the GPU box.

Run:  python oracle/build_ref.py --reference /path/to/xCalibur   (five nvcc builds of ~4 minutes each, run as
parallel processes by ``build_parallel``; ``--only NAME`` builds one)
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SFX = ("-DOKC_PRMTSC=1",)
NAMES = ("tiny", "tiny2", "mid", "main", "program")


def _variants(m):
    """Build name -> the define tuple kernel_fn (or the M = 1 wrapper) passes to _ext for it."""
    return {
        "tiny": tuple(m.TINY_DEFINES) + SFX,
        "tiny2": tuple(m.TINY2_DEFINES) + SFX,
        "mid": tuple(m.MID_DEFINES) + SFX,
        "main": tuple(m.MAIN_FALLBACK_DEFINES) + SFX,
        "program": tuple(m._xc_program_defines()) + SFX,
    }


def source_digest(ref_root: str) -> str:
    path = os.path.join(ref_root, "kernels", "moe_w4a16_h200", "moe_w4a16.py")
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def up_to_date(ref_root: str) -> bool:
    man = os.path.join(OUT, "manifest.json")
    if not os.path.exists(man):
        return False
    with open(man) as f:
        d = json.load(f)
    return d.get("source_sha256") == source_digest(ref_root) and all(
        os.path.exists(os.path.join(OUT, v["so"])) for v in d["builds"].values())


def build(ref_root: str, only=None, verbose: bool = False, manifest_path=None) -> dict:
    """Build the named variants (all when ``only`` is None).  The manifest goes to ``manifest_path`` when given (one
    process's part of a parallel build), else it is merged into oracle/_ref/manifest.json."""
    import torch
    from torch.utils import cpp_extension

    kdir = os.path.join(ref_root, "kernels", "moe_w4a16_h200")
    sys.path.insert(0, kdir)
    try:
        import moe_w4a16 as m
    finally:
        sys.path.remove(kdir)
    os.makedirs(OUT, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="xcb_refbuild_")
    built = {}

    def capture(**kw):
        # the reference's own admission check, appended to every build (the WGS builds carry it already)
        if "xc_admission" not in kw["functions"]:
            kw["cuda_sources"] = kw["cuda_sources"] + m.ADMISSION
            kw["cpp_sources"] = kw["cpp_sources"] + "\nint64_t xc_admission();\n"
            kw["functions"] = list(kw["functions"]) + ["xc_admission"]
        bdir = os.path.join(tmp, kw["name"])
        os.makedirs(bdir, exist_ok=True)
        mod = cpp_extension.load_inline(build_directory=bdir, **{**kw, "verbose": verbose})
        built["last"] = (kw["name"], mod.__file__, list(kw["extra_cuda_cflags"]), list(kw["functions"]))
        return mod

    saved_cap = torch.cuda.get_device_capability
    saved_li = m._xc_load_inline
    torch.cuda.get_device_capability = lambda *a, **k: (10, 0)   # the B200
    m._xc_load_inline = capture
    manifest = {"source_sha256": source_digest(ref_root), "arch": "sm_100", "builds": {}}
    try:
        for name, defines in _variants(m).items():
            if only and name not in only:
                continue
            m._EXTS.pop(tuple(defines) + (("-DOKC_DQ7=1",) if "-DOKC_DQ7=1" not in defines else ()), None)
            m._ext(defines)
            mod_name, so, cflags, fns = built.pop("last")
            dst = f"okc_{name}.so"
            shutil.copyfile(so, os.path.join(OUT, dst))
            manifest["builds"][name] = {"module": mod_name, "so": dst, "defines": list(defines),
                                        "cuda_cflags": cflags, "functions": fns}
            print(f"built {name}: {mod_name}", flush=True)
    finally:
        torch.cuda.get_device_capability = saved_cap
        m._xc_load_inline = saved_li
        shutil.rmtree(tmp, ignore_errors=True)
    if manifest_path:
        with open(manifest_path, "w") as f:
            json.dump(manifest, f, indent=1)
        return manifest
    if only and os.path.exists(os.path.join(OUT, "manifest.json")):
        with open(os.path.join(OUT, "manifest.json")) as f:
            old = json.load(f)
        if old.get("source_sha256") == manifest["source_sha256"]:
            old["builds"].update(manifest["builds"])
            manifest = old
    with open(os.path.join(OUT, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest


def build_parallel(ref_root: str, verbose: bool = False) -> dict:
    """All variants, one process each (the nvcc builds are single-threaded), then one merged manifest."""
    parts = tempfile.mkdtemp(prefix="xcb_refparts_")
    try:
        procs = {}
        for name in NAMES:
            cmd = [sys.executable, os.path.abspath(__file__), "--reference", ref_root, "--only", name,
                   "--manifest", os.path.join(parts, name + ".json")] + (["--verbose"] if verbose else [])
            procs[name] = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        failed = []
        for name, pr in procs.items():
            out, _ = pr.communicate()
            if pr.returncode != 0:
                failed.append(f"{name} (exit {pr.returncode}): {out[-2000:]}")
            else:
                print(out.strip(), flush=True)
        if failed:
            raise RuntimeError("reference builds failed: " + " | ".join(failed))
        manifest = {"source_sha256": source_digest(ref_root), "arch": "sm_100", "builds": {}}
        for name in NAMES:
            with open(os.path.join(parts, name + ".json")) as f:
                manifest["builds"].update(json.load(f)["builds"])
        with open(os.path.join(OUT, "manifest.json"), "w") as f:
            json.dump(manifest, f, indent=1)
        return manifest
    finally:
        shutil.rmtree(parts, ignore_errors=True)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("XCB_REFERENCE", "/root/reference"))
    ap.add_argument("--only", nargs="*", default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--manifest", default=None, help="write this build's manifest here (a parallel build's part)")
    a = ap.parse_args()
    if a.only is None and a.manifest is None:
        build_parallel(a.reference, a.verbose)
    else:
        build(a.reference, a.only, a.verbose, a.manifest)
