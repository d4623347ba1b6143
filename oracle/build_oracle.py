"""Build the CPU oracle (oracle.c -> oracle/liboracle.so) -- TEST INFRASTRUCTURE ONLY.

The oracle is the checker of the B200 kernels; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
load it.  The ggml IQ2_XXS tables are compiled in from the reference's table file by path (B200Q_IQ2_TABLES, else
engine/iq2_tables.inc of the reference checkout: B200Q_REF_ENGINE, else a checkout named "reference" beside this
repository).  Where that file is absent (a GPU box) the prebuilt library is used, and only if it is newer than its
sources: a stale prebuilt library is an error, never silently reused.

With --ref it also builds oracle/_ref/libbolt_ref.so: the reference's own kernels for sm_100a, with oracle/ref_shim.cu
giving them extern "C" entry points.  engine/bolt_kernels.cu compiles from where it lies.  engine/bolt_mma.cu compiles
for sm_100a but for one instruction: the block-scaled fp4 mma.sync of its NVFP4 prompt kernel exists only on sm_120/121,
so the build writes a copy of bolt_mma.cu into the git-ignored oracle/_ref/ with that one asm statement under a
__CUDA_ARCH__ >= 1200 guard (its kernel, mma_nv4_fp4_k, is never called here) and compiles the copy; nothing of the
reference is stored in the repository.  The library lets the GPU tests run libbolt's kernels on the same inputs as
the oracle and the product, and the benchmark's reference arm time them.
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


FP4_ASM = 'asm volatile("mma.sync.aligned.kind::mxf4nvf4'


def guarded_mma_source(src_path, dst_path):
    """bolt_mma.cu with its one sm_12x-only statement (the block-scaled fp4 mma.sync in mma_nv4) under a
    __CUDA_ARCH__ >= 1200 guard, written to dst_path (git-ignored build output)."""
    with open(src_path) as f:
        text = f.read()
    at = text.find(FP4_ASM)
    if at < 0 or text.find(FP4_ASM, at + 1) >= 0:
        raise RuntimeError("bolt_mma.cu: expected exactly one block-scaled fp4 mma.sync statement")
    end = text.find(");", at)
    if end < 0:
        raise RuntimeError("bolt_mma.cu: unterminated fp4 mma.sync statement")
    end += 2
    guarded = (text[:at] + "\n#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 1200\n" + text[at:end] +
               "\n#endif\n" + text[end:])
    with open(dst_path, "w") as f:
        f.write(guarded)
    return dst_path


def build_ref():
    """libbolt's bolt_kernels.cu and (guarded) bolt_mma.cu + oracle/ref_shim.cu for sm_100a ->
    oracle/_ref/libbolt_ref.so."""
    kern = os.path.join(ENGINE, "bolt_kernels.cu")
    mma = os.path.join(ENGINE, "bolt_mma.cu")
    shim = os.path.join(HERE, "ref_shim.cu")
    if not os.path.exists(kern):
        if os.path.exists(REF_OUT) and not _stale(REF_OUT, [shim]):
            return REF_OUT
        return None
    os.makedirs(REF_DIR, exist_ok=True)
    if _stale(REF_OUT, [kern, mma, shim, __file__]):
        mma_copy = guarded_mma_source(mma, os.path.join(REF_DIR, "bolt_mma_sm100.cu"))
        cmd = [NVCC, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
               "-shared", "-Xlinker", "-Bsymbolic", "-diag-suppress", "177", "-I", ENGINE, kern, mma_copy, shim,
               "-o", REF_OUT]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on the reference kernels:\n{r.stderr}")
    return REF_OUT


if __name__ == "__main__":
    print(build())
    if "--ref" in sys.argv:
        print(build_ref())
