"""Build libb200q.so in place: every csrc/*.cu compiled by nvcc for sm_100a (-gencode arch=compute_100a,code=sm_100a)
and linked into one shared library beside this file.

The ggml IQ2_XXS tables are compiled in from the reference's own table file, found by path (B200Q_IQ2_TABLES, else
engine/iq2_tables.inc of a reference checkout named "reference" beside this repository); they are not copied into the
sources.  Where that file is absent (a GPU box), the prebuilt library is used, and only if it is newer than every
source: a stale prebuilt library is an error, never silently reused.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libb200q.so")
OBJ = os.path.join(HERE, "_build")
TABLES = os.environ.get("B200Q_IQ2_TABLES",
                        os.path.join(os.path.dirname(ROOT), "reference", "engine", "iq2_tables.inc"))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", f"-DB200Q_IQ2_TABLES=\"{TABLES}\"", "-I", os.path.join(ROOT, "include")]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _all_sources():
    inc = os.path.join(ROOT, "include")
    return (sources() + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))] +
            [os.path.join(inc, h) for h in os.listdir(inc) if h.endswith(".h")])


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose=False):
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    inc = os.path.join(ROOT, "include")
    headers += [os.path.join(inc, h) for h in os.listdir(inc) if h.endswith(".h")]
    if not _stale(obj, [src, __file__] + headers):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force=False, verbose=False):
    """Compile and link libb200q.so; returns its path."""
    if not os.path.exists(TABLES):
        if os.path.exists(OUT) and not _stale(OUT, _all_sources()):
            return OUT
        raise RuntimeError(f"IQ2_XXS table file not found at {TABLES} and no prebuilt {OUT} newer than its sources")
    os.makedirs(OBJ, exist_ok=True)
    if force:
        for f in os.listdir(OBJ):
            os.remove(os.path.join(OBJ, f))
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if force or _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
