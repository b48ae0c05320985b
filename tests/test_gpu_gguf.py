"""A MoE layer loaded from a GGUF file matches the oracle on the same bytes.

The synthetic layer's tensors are written into a GGUF file under the names the
reference loads (src/gemma4.rs:378-406 for the fused Gemma experts; the llama.cpp names
for separate gate / up / down experts with a shared expert), read back through the GGUF
index and expert layout (include/diskmule_gguf.h), mapped to the device, and the layer's
forward is checked against the oracle run on the synthetic bytes.
"""
import numpy as np
import pytest

from diskmule_b200 import _native as N
from diskmule_b200.gguf import TensorSource, moe_layer_from_gguf, write_gguf
from diskmule_b200.moe import CudaContext
from diskmule_b200.synthetic import SyntheticLayer, input_spec, layer_specs, vectors

from test_gpu_parity import check, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = CudaContext(0)
    yield c
    c.close()


def _gguf_tensors(name, cfg, specs, vecs, block=0):
    H, I, E = cfg["hidden"], cfg["intermediate"], cfg["experts"]
    p = f"blk.{block}."
    t = [(p + "ffn_gate_inp.weight", [H, E], N.F32, specs["router"].host().tobytes())]
    if cfg["family"] == "gemma4":
        t += [(p + "ffn_gate_inp.scale", [H], N.F32, vecs["router_scale"].tobytes()),
              (p + "pre_ffw_norm_2.weight", [H], N.F32, vecs["routed_pre_norm"].tobytes()),
              (p + "ffn_gate_up_exps.weight", [H, 2 * I, E], cfg["gate_type"],
               specs["gate"].host().tobytes()),
              (p + "ffn_down_exps.weight", [I, H, E], cfg["down_type"], specs["down"].host().tobytes()),
              (p + "ffn_down_exps.scale", [E], N.F32, vecs["expert_scale"].tobytes())]
    else:
        t += [(p + "ffn_gate_exps.weight", [H, I, E], cfg["gate_type"], specs["gate"].host().tobytes()),
              (p + "ffn_up_exps.weight", [H, I, E], cfg["gate_type"], specs["up"].host().tobytes()),
              (p + "ffn_down_exps.weight", [I, H, E], cfg["down_type"], specs["down"].host().tobytes()),
              (p + "ffn_gate_shexp.weight", [H, I], cfg["gate_type"], specs["shared_gate"].host().tobytes()),
              (p + "ffn_up_shexp.weight", [H, I], cfg["gate_type"], specs["shared_up"].host().tobytes()),
              (p + "ffn_down_shexp.weight", [I, H], cfg["down_type"],
               specs["shared_down"].host().tobytes()),
              (p + "ffn_gate_inp_shexp.weight", [H], N.F32,
               specs["shared_gate_vector"].host().tobytes())]
    return t


@pytest.mark.parametrize("name,T", [("gemma4-small", 24), ("qwen35-small", 40), ("qwen35-small", 3)])
def test_layer_from_gguf_matches_the_oracle(ctx, tmp_path, name, T):
    from diskmule_b200.synthetic import CONFIGS
    cfg = dict(CONFIGS[name])
    specs, vecs = layer_specs(cfg, 6), vectors(cfg, 6)
    path = tmp_path / f"{name}.gguf"
    write_gguf(str(path), {"general.architecture": (8, cfg["family"])},
               _gguf_tensors(name, cfg, specs, vecs, block=3))
    src = TensorSource.open(str(path))
    gl = moe_layer_from_gguf(ctx, src, 3, cfg["family"], cfg["top_k"],
                             epsilon=cfg.get("epsilon", 1e-6))
    try:
        assert gl.layout.expert_count == cfg["experts"]
        assert gl.layout.down_bytes == specs["down"].expert_bytes
        x = input_spec(cfg, T, 9).host().view(np.float32).reshape(T, -1)
        y, idx, w = gl.layer.forward_host(x)
        ref = SyntheticLayer(name, cfg, 6, None, specs, vecs)
        y_ref, idx_ref, w_ref = run_oracle(ref, x)
        check(y, idx, w, y_ref, idx_ref, w_ref)
    finally:
        gl.close()
        src.close()
