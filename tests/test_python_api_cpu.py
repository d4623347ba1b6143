"""CPU tests of the Python operator mirror (b200q.py): no CPU fallback.  Every operator refuses host tensors with
B200QError before anything reaches the C ABI, whichever operand is on the host, so no host address can reach a
kernel; and a missing library is an error."""
import os

import pytest
import torch

import b200q

N, K = 32, 256


def cpu(*shape, dtype=torch.uint8):
    return torch.zeros(*shape, dtype=dtype)


CASES = {
    "repack_iq2": lambda: b200q.repack_iq2(cpu(N * K // 256 * 66), N, K),
    "k_quant_rows": lambda: b200q.k_quant_rows(cpu(4, K, dtype=torch.float32)),
    "k_route": lambda: b200q.k_route(cpu(4, 16, dtype=torch.float32), 2),
    "k_moe_group": lambda: b200q.k_moe_group(cpu(8, dtype=torch.int32), 16),
    "k_combine": lambda: b200q.k_combine(cpu(8, K, dtype=torch.float32), cpu(4, 2, dtype=torch.float32), 2),
    "mma_iq2": lambda: b200q.mma_iq2(cpu(N * K // 256 * 66), N, K, cpu(2, K, dtype=torch.int8),
                                     cpu(2, K // 32, dtype=torch.float32)),
    "moe_up (host slab and tables)": lambda: b200q.moe_up(cpu(64), 2, N, K, cpu(2, dtype=torch.int32),
                                                          cpu(3, dtype=torch.int32), cpu(4, dtype=torch.int32), 2,
                                                          cpu(2, K, dtype=torch.int8), cpu(2, 8, dtype=torch.float32)),
    "tile_nv4": lambda: b200q.tile_nv4(cpu(N, K // 2), cpu(N, K // 16), N, K),
    "tile_q8": lambda: b200q.tile_q8(cpu(N, K // 32 * 34), N, K),
    "mma_nv4": lambda: b200q.mma_nv4(cpu(1024), 1.0, N, K, cpu(1, K, dtype=torch.float32)),
    "mma_q8": lambda: b200q.mma_q8(cpu(1024), N, K, cpu(1, K, dtype=torch.float32)),
    "quant_nv4_rows": lambda: b200q.quant_nv4_rows(cpu(4, K, dtype=torch.float32)),
    "moe_prompt": lambda: b200q.moe_prompt(cpu(64), cpu(64), 2, K, K, cpu(2, dtype=torch.int32), cpu(3, dtype=torch.int32),
                                           cpu(4, dtype=torch.int32), 2, cpu(2, K, dtype=torch.float32)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_host_operands_are_refused(name):
    with pytest.raises(b200q.B200QError) as e:
        CASES[name]()
    assert e.value.args and "CUDA tensor" in str(e.value)


def test_missing_library_is_an_error(monkeypatch):
    monkeypatch.setattr(b200q, "LIB_PATH", os.path.join(os.path.dirname(b200q.LIB_PATH), "no_such_libb200q.so"))
    monkeypatch.setattr(b200q, "_LIB", None)
    with pytest.raises(RuntimeError, match="missing"):
        b200q.lib()
