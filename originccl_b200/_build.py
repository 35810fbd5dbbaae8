"""Native build of the library: csrc/ -> originccl_b200/_lib/libbccl.so (+ the bccl_run launcher).

Kernels are compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``); host C++
is compiled with g++. A small ninja file is generated so rebuilds are incremental and use every
core. nvcc cross-compiles without a GPU, so this runs on CPU-only machines as well.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "csrc"
LIBDIR = ROOT / "originccl_b200" / "_lib"
BUILD = ROOT / "build" / "native"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = "-gencode arch=compute_100a,code=sm_100a"


def _site_packages() -> Path:
    return Path(sysconfig.get_paths()["purelib"])


def nccl_include() -> Path | None:
    p = _site_packages() / "nvidia" / "nccl" / "include"
    return p if (p / "nccl.h").exists() else None


def cutlass_include() -> Path | None:
    for rel in ("flashinfer/data/cutlass/include", "tilelang/3rdparty/cutlass/include"):
        p = _site_packages() / rel
        if (p / "cute").exists():
            return p
    return None


# Host sources whose inner loops must be vectorised (-O2's cost model leaves loops with a
# run-time trip count scalar).
VECTORIZED = {"host_reduce.cc"}


def _sources() -> tuple[list[Path], list[Path]]:
    cc = sorted(p for p in CSRC.rglob("*.cc") if not {"launcher", "examples"} & set(p.parts))
    cu = sorted(CSRC.rglob("*.cu"))
    return cc, cu


def _ninja_file() -> str:
    cc, cu = _sources()
    nccl = nccl_include()
    incs = f"-I{CSRC} -I{CSRC / 'include'} -I{CUDA_HOME / 'include'}"
    if nccl:
        incs += f" -I{nccl}"
    cxxflags = f"-O2 -g -std=c++17 -fPIC -Wall -Wextra -Wno-unused-parameter -Wno-missing-field-initializers {incs}"
    nvflags = (f"{ARCH} -lineinfo -O3 -std=c++17 -Xcompiler -fPIC --expt-relaxed-constexpr "
               f"-Xptxas -warn-spills {incs}")
    lines = [
        "ninja_required_version = 1.5",
        f"cxx = g++",
        f"nvcc = {CUDA_HOME / 'bin' / 'nvcc'}",
        f"cxxflags = {cxxflags}",
        f"nvflags = {nvflags}",
        "rule cxx",
        "  command = $cxx -MMD -MF $out.d $cxxflags -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $out",
        "rule nvcc",
        "  command = $nvcc -MD -MF $out.d $nvflags -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $out",
        "rule link",
        f"  command = $nvcc {ARCH} -shared -cudart static -o $out.tmp $in -ldl -lpthread -lrt && mv -f $out.tmp $out",
        "  description = LINK $out",
        "rule linkexe",
        "  command = $cxx -o $out.tmp $in -lpthread && mv -f $out.tmp $out",
        "  description = LINK $out",
        "rule cc",
        f"  command = gcc -MMD -MF $out.d -O2 -g -std=c11 -Wall -Wextra -pedantic -I{CSRC / 'include'} -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CC $out",
        "rule linkexample",
        f"  command = $cxx -o $out.tmp $in -L{LIBDIR} -lbccl -Wl,-rpath,'$$ORIGIN' -L{CUDA_HOME / 'lib64'} -lcudart "
        f"-Wl,-rpath,{CUDA_HOME / 'lib64'} -lpthread && mv -f $out.tmp $out",
        "  description = LINK $out",
    ]
    objs = []
    for src in cc:
        obj = BUILD / (str(src.relative_to(CSRC)).replace("/", "_") + ".o")
        lines.append(f"build {obj}: cxx {src}")
        if src.name in VECTORIZED:
            lines.append("  cxxflags = $cxxflags -O3")
        objs.append(obj)
    for src in cu:
        obj = BUILD / (str(src.relative_to(CSRC)).replace("/", "_") + ".o")
        lines.append(f"build {obj}: nvcc {src}")
        objs.append(obj)
    lines.append(f"build {LIBDIR / 'libbccl.so'}: link {' '.join(map(str, objs))}")
    launcher = CSRC / "launcher" / "bccl_run.cc"
    lobj = BUILD / "launcher_bccl_run.cc.o"
    lines.append(f"build {lobj}: cxx {launcher}")
    lines.append(f"build {LIBDIR / 'bccl_run'}: linkexe {lobj}")
    for ex in sorted((CSRC / "examples").glob("*.cc")):
        eobj = BUILD / f"examples_{ex.name}.o"
        lines.append(f"build {eobj}: cxx {ex}")
        lines.append(f"build {LIBDIR / ex.stem}: linkexample {eobj} | {LIBDIR / 'libbccl.so'}")
    for ex in sorted((CSRC / "examples").glob("*.c")):  # C callers of the C interface
        eobj = BUILD / f"examples_{ex.name}.o"
        lines.append(f"build {eobj}: cc {ex}")
        lines.append(f"build {LIBDIR / ex.stem}: linkexample {eobj} | {LIBDIR / 'libbccl.so'}")
    return "\n".join(lines) + "\n"


SANITIZERS = {
    "asan": "-fsanitize=address,undefined -fno-sanitize-recover=undefined -fno-omit-frame-pointer",
    "tsan": "-fsanitize=thread -fno-omit-frame-pointer",
}


def _sanitized_ninja_file(kind: str) -> str:
    """Host C++ of the library, the launcher and the examples rebuilt with a sanitizer; the CUDA
    objects of the regular build are linked in unchanged (kernels are not instrumented)."""
    cc, cu = _sources()
    out = ROOT / "build" / f"san-{kind}"
    nccl = nccl_include()
    incs = f"-I{CSRC} -I{CSRC / 'include'} -I{CUDA_HOME / 'include'}"
    if nccl:
        incs += f" -I{nccl}"
    san = SANITIZERS[kind]
    cxxflags = f"-O1 -g -std=c++17 -fPIC -Wall -Wno-unused-parameter -Wno-missing-field-initializers {san} {incs}"
    lines = [
        "ninja_required_version = 1.5",
        f"cxxflags = {cxxflags}",
        "rule cxx",
        "  command = g++ -MMD -MF $out.d $cxxflags -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $out",
        "rule link",
        f"  command = g++ {san} -shared -o $out.tmp $in -L{CUDA_HOME / 'lib64'} -lcudart_static -ldl -lpthread -lrt "
        "&& mv -f $out.tmp $out",
        "  description = LINK $out",
        "rule linkexe",
        f"  command = g++ {san} -o $out.tmp $in -L{out} -lbccl -Wl,-rpath,'$$ORIGIN' -L{CUDA_HOME / 'lib64'} "
        f"-lcudart -Wl,-rpath,{CUDA_HOME / 'lib64'} -lpthread && mv -f $out.tmp $out",
        "  description = LINK $out",
    ]
    objs = []
    for src in cc:
        obj = out / (str(src.relative_to(CSRC)).replace("/", "_") + ".o")
        lines.append(f"build {obj}: cxx {src}")
        if src.name in VECTORIZED:
            lines.append("  cxxflags = $cxxflags -O3")
        objs.append(str(obj))
    objs += [str(BUILD / (str(src.relative_to(CSRC)).replace("/", "_") + ".o")) for src in cu]
    lines.append(f"build {out / 'libbccl.so'}: link {' '.join(objs)}")
    for ex in sorted((CSRC / "examples").glob("*.cc")):
        eobj = out / f"examples_{ex.name}.o"
        lines.append(f"build {eobj}: cxx {ex}")
        lines.append(f"build {out / ex.stem}: linkexe {eobj} | {out / 'libbccl.so'}")
    return "\n".join(lines) + "\n"


class _BuildLock:
    """Serialises builds across processes (pytest-xdist workers may build at the same time). Links
    write a temporary file and rename it into place, so a process that loads a library or program
    while another relinks it sees the old or the new file, never a half-written one."""

    def __enter__(self):
        import fcntl
        (ROOT / "build").mkdir(parents=True, exist_ok=True)
        self._f = open(ROOT / "build" / ".lock", "w")
        fcntl.flock(self._f, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        import fcntl
        fcntl.flock(self._f, fcntl.LOCK_UN)
        self._f.close()


def build_sanitized(kind: str, verbose: bool = False) -> Path:
    """Builds libbccl.so and the example programs (bccl_check, bccl_transport_check) with
    AddressSanitizer + UndefinedBehaviorSanitizer (``"asan"``) or ThreadSanitizer (``"tsan"``)
    into build/san-<kind>/ and returns that folder. Used by the CPU tests of the host path; run
    the programs under the regular ``bccl_run`` launcher."""
    if kind not in SANITIZERS:
        raise ValueError(f"unknown sanitizer {kind!r} (asan, tsan)")
    build(verbose)  # the CUDA objects are shared with the regular build
    with _BuildLock():
        return _build_sanitized_locked(kind, verbose)


def _build_sanitized_locked(kind: str, verbose: bool) -> Path:
    out = ROOT / "build" / f"san-{kind}"
    out.mkdir(parents=True, exist_ok=True)
    ninja_path = out / "build.ninja"
    content = _sanitized_ninja_file(kind)
    if not ninja_path.exists() or ninja_path.read_text() != content:
        ninja_path.write_text(content)
    ninja = shutil.which("ninja") or str(Path(sys.executable).parent / "ninja")
    res = subprocess.run([ninja, "-C", str(out)] + (["-v"] if verbose else []), capture_output=not verbose,
                         text=True)
    if res.returncode != 0:
        raise RuntimeError(f"sanitized build ({kind}) failed:\n{((res.stdout or '') + (res.stderr or ''))[-8000:]}")
    return out


def build(verbose: bool = False) -> Path:
    """Compiles everything (incrementally) and returns the path of libbccl.so."""
    with _BuildLock():
        return _build_locked(verbose)


def _build_locked(verbose: bool) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    ninja_path = BUILD / "build.ninja"
    content = _ninja_file()
    if not ninja_path.exists() or ninja_path.read_text() != content:
        ninja_path.write_text(content)
    ninja = shutil.which("ninja") or str(Path(sys.executable).parent / "ninja")
    cmd = [ninja, "-C", str(BUILD)]
    if verbose:
        cmd.append("-v")
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        out = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError(f"native build failed:\n{out[-8000:]}")
    return LIBDIR / "libbccl.so"


def ptxas_report() -> list[dict]:
    """Registers, spills, stack and static shared memory of every kernel, from ``ptxas -v`` on
    each CUDA source compiled with the library's own flags (the object is thrown away). Returns
    one dict per kernel entry: file, kernel (demangled), registers, spill_stores, spill_loads,
    stack, smem."""
    import re
    import tempfile
    _, cu = _sources()
    nccl = nccl_include()
    incs = [f"-I{CSRC}", f"-I{CSRC / 'include'}", f"-I{CUDA_HOME / 'include'}"] + ([f"-I{nccl}"] if nccl else [])
    rows = []
    with tempfile.TemporaryDirectory() as td:
        for src in cu:
            cmd = [str(CUDA_HOME / "bin" / "nvcc"), *ARCH.split(), "-lineinfo", "-O3", "-std=c++17",
                   "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-v", *incs,
                   "-c", str(src), "-o", os.path.join(td, "k.o")]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n{res.stderr[-4000:]}")
            cur = None
            for line in res.stderr.splitlines():
                m = re.search(r"Compiling entry function '([^']+)'", line)
                if m:
                    cur = {"file": str(src.relative_to(ROOT)), "mangled": m.group(1), "registers": 0,
                           "spill_stores": 0, "spill_loads": 0, "stack": 0, "smem": 0}
                    rows.append(cur)
                    continue
                if cur is None:
                    continue
                m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
                if m:
                    cur["stack"], cur["spill_stores"], cur["spill_loads"] = map(int, m.groups())
                m = re.search(r"Used (\d+) registers", line)
                if m:
                    cur["registers"] = int(m.group(1))
                m = re.search(r"(\d+) bytes smem", line)
                if m:
                    cur["smem"] = int(m.group(1))
    names = subprocess.run(["c++filt"], input="\n".join(r["mangled"] for r in rows), capture_output=True,
                           text=True).stdout.splitlines() if shutil.which("c++filt") else []
    for i, r in enumerate(rows):
        r["kernel"] = names[i] if i < len(names) else r["mangled"]
        del r["mangled"]
    return rows


if __name__ == "__main__":
    if "--ptxas-report" in sys.argv:
        print("| file | kernel | registers | spill stores | spill loads | stack | static smem |")
        print("|---|---|---|---|---|---|---|")
        for r in ptxas_report():
            k = r["kernel"].replace("|", "\\|")
            k = k if len(k) <= 150 else k[:147] + "..."
            print(f"| {r['file']} | `{k}` | {r['registers']} | {r['spill_stores']} | {r['spill_loads']} | "
                  f"{r['stack']} | {r['smem']} |")
        sys.exit(0)
    kinds = [a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--sanitize=")]
    for k in kinds:
        print(build_sanitized(k, verbose="-v" in sys.argv))
    if not kinds:
        print(build(verbose="-v" in sys.argv))
