"""Gemma 4's whole feed-forward block on the GPU against the oracle.

The oracle restates src/gemma4/cpu.rs:547-620 for each token: the dense shared FFN on
rms_norm(x, feed_forward_norm) and its post norm, the routed branch and its post norm,
their sum through the post feed-forward norm, the residual add and the layer output
scale. Selections must be bit-exact; the block output within the 1e-3 relative-L2 bar.
"""
import numpy as np
import pytest
import torch

from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import build_gemma_block, input_spec
from oracle import oracle as O

from test_gpu_parity import check

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


@pytest.mark.parametrize("name,T", [("gemma4-small", 1), ("gemma4-small", 48),
                                    ("gemma4-small-q8", 7), ("gemma4", 3)])
def test_gemma_block_matches_the_oracle(ctx, name, T):
    gb = build_gemma_block(ctx, name, seed=4)
    try:
        cfg = gb.sl.cfg
        H, k = cfg["hidden"], cfg["top_k"]
        x = input_spec(cfg, T, 17).host().view(np.float32).reshape(T, H)
        xd = torch.from_numpy(x.copy()).cuda()
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        i = torch.empty((T, k), dtype=torch.int32, device="cuda")
        w = torch.empty((T, k), dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        gb.block.forward(xd.data_ptr(), y.data_ptr(), T, i.data_ptr(), w.data_ptr(), stream)
        gb.block.status(stream)
        idx = i.cpu().numpy().view(np.uint32)
        experts = sorted(set(idx.ravel().tolist()))
        rc, y_ref, idx_ref, w_ref = O.gemma_ffn_block(gb.sl.host_weights(experts), gb.host_ffn(),
                                                      x, threads=8)
        assert rc == O.OK
        check(y.cpu().numpy(), idx, w.cpu().numpy(), y_ref, idx_ref, w_ref)
    finally:
        gb.close()
