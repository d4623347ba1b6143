"""Build tests/_build/libbolt_shim_harness.so (TEST INFRASTRUCTURE): tests/bolt_shim_harness.cu linked against the
package's libb200q.so (nvcc, sm_100a host code only; the shims it calls live in libb200q).  Where nvcc or the
library is missing (a GPU box with the prebuilt files), an existing build is kept if it is newer than its source."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "nemotron-3.5-bolt-tensorfold-dgx-spark_b200")
SRC = os.path.join(HERE, "bolt_shim_harness.cu")
OUT = os.path.join(HERE, "_build", "libbolt_shim_harness.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def build():
    lib = os.path.join(PKG, "libb200q.so")
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(SRC), os.path.getmtime(lib)):
        return OUT
    if not os.path.exists(NVCC):
        if os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
            return OUT
        raise RuntimeError("nvcc not found and no prebuilt harness newer than its source")
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I", os.path.join(ROOT, "include"), SRC, "-o", OUT, "-L", PKG, "-lb200q",
           "-Xlinker", "-rpath=$ORIGIN/../../nemotron-3.5-bolt-tensorfold-dgx-spark_b200"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"harness build failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build())
