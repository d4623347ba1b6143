"""The Q8_0 GEMMs at the model's lm_head shape (131072 x 4096, engine/bolt_host.cu:730,933) and row counts: decode
rows (M = 1 and 16, the t16 decode GEMV, libbolt's mma_q8 at decode) and verify windows (M = 128 and a ragged 100, the
tcgen05 prompt GEMM, where libbolt's K-split decode rule takes verify rows, bolt_mma.cu:1115-1118).

The scalar oracle over all 131072 outputs is too slow for a test, so it runs on 1024 seeded output rows of the matrix
(their blocks, the same x): bars as for the other Q8_0 GEMMs, 1e-5 relative L2 against the exact arithmetic for the
decode GEMV (exact operands, fp32 sums) and 1e-4 against the fp16 fold for the prompt GEMM, plus BASELINE's tolerance
against the exact arithmetic."""
import numpy as np
import pytest
import torch

import b200q
import oracle as O
from helpers import assert_tolerance, normal_bf16, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"
N, K = 131072, 4096


@pytest.fixture(scope="module")
def lm_head():
    r = np.random.default_rng(131)
    qv = r.integers(-127, 128, (N, K // 32, 32), dtype=np.int8)
    d = r.uniform(1e-3, 1e-2, (N, K // 32)).astype(np.float16)
    blocks = np.concatenate([d.view(np.uint8).reshape(N, K // 32, 2), qv.view(np.uint8)], -1)
    raw = torch.from_numpy(blocks.reshape(-1)).to(DEV)
    w16 = b200q.tile_q8(raw, N, K)
    wtc = b200q.tile_q8_tc(raw, N, K)
    del raw
    sub = np.sort(np.random.default_rng(132).choice(N, 1024, replace=False))
    return w16, wtc, blocks[sub].reshape(len(sub), -1), sub


@pytest.mark.parametrize("M", [1, 16])
def test_lm_head_decode_rows(lm_head, M):
    w16, _, sub_blocks, sub = lm_head
    xb, x = normal_bf16(M, (M, K))   # bf16 rows: exact in the GEMV's fp16 operands
    y = b200q.mma_q8(w16, N, K, torch.from_numpy(xb).to(DEV).view(torch.bfloat16)).cpu().numpy()
    assert b200q.device_error() == 0
    ref = O.q8_gemm_exact(sub_blocks, len(sub), K, x)
    assert rel_l2(y[:, sub], ref) < 1e-5
    assert np.isfinite(y).all()


@pytest.mark.parametrize("M", [128, 100])
def test_lm_head_verify_rows(lm_head, M):
    _, wtc, sub_blocks, sub = lm_head
    xb, x = normal_bf16(1000 + M, (M, K))
    y = b200q.mma_q8_prompt(wtc, N, K, torch.from_numpy(xb).to(DEV).view(torch.bfloat16)).cpu().numpy()
    assert b200q.device_error() == 0
    assert rel_l2(y[:, sub], O.q8_gemm_f16fold(sub_blocks, len(sub), K, x)) < 1e-4
    assert_tolerance(y[:, sub], O.q8_gemm_exact(sub_blocks, len(sub), K, x))
    assert np.isfinite(y).all()
