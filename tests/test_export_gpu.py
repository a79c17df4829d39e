"""A standalone export (moss_tts_lite/export.py:691-770) loaded by this
package decodes bit for bit like GptqMossTTS fed the same state, and within
bf16 noise of the reference's own load_standalone_model on the directory."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from test_export_cpu import make_standalone
from test_gptq_gpu import NAMES, _state
from test_step_gpu import SMALL, _prompt, _t, _torch_weights, _weights

pytestmark = pytest.mark.gpu


def test_standalone_export_decode(tmp_path):
    dev = require_cuda()
    ref_gptq = pytest.importorskip("moss_tts_lite.gptq")
    ref_export = pytest.importorskip("moss_tts_lite.export")
    from moss_tts_lite_b200.export import load_standalone_model
    from moss_tts_lite_b200.gptq import GptqMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    w = _weights(seed=91)
    tw = _torch_weights(w, dev)
    gmap = {(0, "o"): 64}
    keep = [(1, "down")]
    state = _state(tw, ref_gptq, gmap, {(1, "down")})
    # the export carries every non-payload weight, plus the kept projection
    base = {k: v.cpu() for k, v in tw.items()
            if not any(k == f"language_model.layers.{li}.{key}.weight" for li in state for key in NAMES.values())}
    base["language_model.layers.1.mlp.down_proj.weight"] = tw["language_model.layers.1.mlp.down_proj.weight"].cpu()
    H, D = SMALL["hidden"], SMALL["head_dim"]
    cfg = {"layer0_q_proj_shape": [SMALL["n_heads"] * D, H], "layer0_k_proj_shape": [SMALL["n_kv"] * D, H]}
    make_standalone(str(tmp_path), base, state, gmap, keep, cfg)
    _, mine = load_standalone_model(str(tmp_path), device=dev, max_seq_len=64)
    direct = GptqMossTTS(MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=64), state, bf16_keep=keep,
                         group_size_map=gmap)
    _, ref = ref_export.load_standalone_model(str(tmp_path), device=dev, max_seq_len=64)
    ids = _t(_prompt(8, seed=92), dev).view(1, 8, 33)
    for f in (mine, direct, ref):
        f.prefill(ids)
        f.capture()
    rng = np.random.default_rng(93)
    for t in range(4):
        row = _t(np.concatenate([[151656], rng.integers(0, 1024, 32)]).astype(np.int64), dev).view(1, 33)
        a = [x.clone() for x in mine.step(row, 8 + t, audio2=True)[1:]]
        b = [x.clone() for x in direct.step(row, 8 + t, audio2=True)[1:]]
        r = [x.float().clone() for x in ref.step(row, 8 + t, audio2=True)[1:]]
        for x, y in zip(a, b):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16)), t
        rel = float((a[1].float() - r[1]).norm() / r[1].norm())
        assert rel < 2e-2, (t, rel)
