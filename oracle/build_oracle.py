"""Build the CPU oracle (oracle.c -> oracle/liboracle.so) -- TEST INFRASTRUCTURE ONLY.

The oracle is the checker of the B200 kernels; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
load it.  The ggml IQ2_XXS tables are compiled in from the reference's table file by path (B200Q_IQ2_TABLES, else
engine/iq2_tables.inc of the reference checkout: B200Q_REF_ENGINE, else a checkout named "reference" beside this
repository).  Where that file is absent (a GPU box) the prebuilt library is used, and only if it is newer than its
sources: a stale prebuilt library is an error, never silently reused.

With --ref it also builds oracle/_ref/libbolt_ref.so: the reference's own kernels (engine/bolt_kernels.cu, compiled
from where it lies) for sm_100a, with oracle/ref_shim.cu giving them extern "C" entry points.  That library lets the
GPU tests run libbolt's kernels on the same inputs as the oracle and the product.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_OUT = os.path.join(REF_DIR, "libbolt_ref.so")
ENGINE = os.environ.get("B200Q_REF_ENGINE",
                        os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "engine"))
TABLES = os.environ.get("B200Q_IQ2_TABLES", os.path.join(ENGINE, "iq2_tables.inc"))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _stale(target, deps):
    return not os.path.exists(target) or any(os.path.getmtime(d) > os.path.getmtime(target) for d in deps)


def build():
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(TABLES):
        if os.path.exists(OUT) and not _stale(OUT, [src]):
            return OUT
        raise RuntimeError(f"IQ2_XXS table file not found at {TABLES} and no up-to-date prebuilt {OUT}")
    if _stale(OUT, [src, __file__]):
        cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared",
               f"-DB200Q_IQ2_TABLES=\"{TABLES}\"", src, "-o", OUT, "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"gcc failed:\n{r.stderr}")
    return OUT


def build_ref():
    """libbolt's bolt_kernels.cu + oracle/ref_shim.cu for sm_100a -> oracle/_ref/libbolt_ref.so."""
    kern = os.path.join(ENGINE, "bolt_kernels.cu")
    shim = os.path.join(HERE, "ref_shim.cu")
    if not os.path.exists(kern):
        if os.path.exists(REF_OUT) and not _stale(REF_OUT, [shim]):
            return REF_OUT
        return None
    os.makedirs(REF_DIR, exist_ok=True)
    if _stale(REF_OUT, [kern, shim, __file__]):
        cmd = [NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
               "-shared", "-I", ENGINE, kern, shim, "-o", REF_OUT]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on the reference kernels:\n{r.stderr}")
    return REF_OUT


if __name__ == "__main__":
    print(build())
    if "--ref" in sys.argv:
        print(build_ref())
