import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nemotron-3.5-bolt-tensorfold-dgx-spark_b200")
for p in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "oracle"), PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")
    # tmp_path directories (the checkpoint tests' shards) stay inside the repository, under the ignored tests/_build
    if not config.option.basetemp:
        config.option.basetemp = os.path.join(ROOT, "tests", "_build", "tmp")
