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
    if os.path.exists(dst_path):   # unchanged: keep its time stamp, so what is built from it is not rebuilt
        with open(dst_path) as f:
            if f.read() == guarded:
                return dst_path
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


LINK_OUT = os.path.join(REF_DIR, "libbolt_b200.so")
PKG = os.path.join(os.path.dirname(HERE), "nemotron-3.5-bolt-tensorfold-dgx-spark_b200")


def build_bolt_link():
    """libbolt as a whole, with its hot path from this engine: the reference's own engine/bolt_host.cu, bolt_kernels.cu,
    bolt_draft.cu and (guarded) bolt_mma.cu compiled for sm_100a, every launcher that libb200q.so also defines (its
    libbolt-signature shims, include/b200q_bolt.h) made local to the reference's objects (objcopy --localize-symbol),
    and the result linked against libb200q.so -> oracle/_ref/libbolt_b200.so.  bolt_host.cu's calls of those launchers
    are then undefined in the link and bound to libb200q.so at load time; the rest of libbolt (the Mamba scan,
    attention, the drafter, the host logic behind the 45 exports of engine/bolt.def) is the reference's.  Returns the
    path, or None where the reference checkout is absent."""
    srcs = {n: os.path.join(ENGINE, n + ".cu") for n in ("bolt_host", "bolt_kernels", "bolt_draft")}
    if not all(os.path.exists(v) for v in srcs.values()):
        return LINK_OUT if os.path.exists(LINK_OUT) else None
    lib = os.path.join(PKG, "libb200q.so")
    obj_dir = os.path.join(REF_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    srcs["bolt_mma"] = guarded_mma_source(os.path.join(ENGINE, "bolt_mma.cu"), os.path.join(REF_DIR, "bolt_mma_sm100.cu"))
    objs = {}
    import concurrent.futures

    def compile_one(item):
        name, src = item
        obj = os.path.join(obj_dir, name + ".o")
        if _stale(obj, [src, __file__]):
            cmd = [NVCC, "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
                   "-diag-suppress", "177", "-I", ENGINE, "-c", src, "-o", obj]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return name, obj
    with concurrent.futures.ThreadPoolExecutor(4) as ex:
        objs = dict(ex.map(compile_one, srcs.items()))
    if not _stale(LINK_OUT, list(objs.values()) + [lib, __file__]):
        return LINK_OUT
    shims = set(_defined(lib)) - {x for x in _defined(lib) if x.startswith("b200q_")}
    linked = [objs["bolt_host"], objs["bolt_draft"]]
    for name in ("bolt_kernels", "bolt_mma"):
        mine = sorted(shims & set(_defined(objs[name])))
        out = os.path.join(obj_dir, name + ".local.o")
        r = subprocess.run(["objcopy", *[f"--localize-symbol={x}" for x in mine], objs[name], out],
                           capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"objcopy failed on {name}:\n{r.stderr}")
        linked.append(out)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LINK_OUT, *linked, "-L", PKG, "-lb200q",
           "-lcuda", "-Xlinker", "-rpath=$ORIGIN/../../nemotron-3.5-bolt-tensorfold-dgx-spark_b200"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    return LINK_OUT


def _defined(path):
    """the global text symbols an object or library defines (mangled)"""
    dyn = ["-D"] if path.endswith(".so") else []
    r = subprocess.run(["nm", *dyn, "--defined-only", path], capture_output=True, text=True, check=True)
    return [f[2] for f in (l.split() for l in r.stdout.splitlines()) if len(f) == 3 and f[1] == "T"]


if __name__ == "__main__":
    print(build())
    if "--ref" in sys.argv:
        print(build_ref())
    if "--link" in sys.argv:
        print(build_bolt_link())
