"""The reference-side ctypes shim (moss_tts_lite_b200/ref_shim.py, the
binding INTEGRATION.md documents) installed into the reference's own
FastMossTTS: its _quantize packs with mtl_w4_pack_ref and its _linear calls
mtl_w4a16_linear, while the reference keeps its graphs, eager attention and
prefill.  Checked like the reference's phase 0 (tests/test_fast.py:57-93):
graph replay equals the reference's eager pass bit for bit; and against
the unshimmed reference (tinygemm) the decode agrees within bf16 noise."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from test_step_gpu import _prompt, _t, _torch_weights, _weights

pytestmark = pytest.mark.gpu


def test_shim_phase0_graph_equals_eager_and_tinygemm():
    dev = require_cuda()
    ref_fast = pytest.importorskip("moss_tts_lite.fast")
    ref_model = pytest.importorskip("moss_tts_lite.model")
    from moss_tts_lite_b200 import ref_shim
    Shim = ref_shim.install(ref_fast.FastMossTTS)
    w = _weights(seed=71)
    fast = Shim(ref_model.MossTTSModel(_torch_weights(w, dev), device=dev, dtype=torch.bfloat16, max_seq_len=64),
                quant="w4")
    base = ref_fast.FastMossTTS(ref_model.MossTTSModel(_torch_weights(w, dev), device=dev, dtype=torch.bfloat16,
                                                       max_seq_len=64), quant="w4")
    assert isinstance(fast.qlayers[0]["q"][0], torch.Tensor) and fast.qlayers[0]["q"][0].dtype == torch.uint8
    ids = _t(_prompt(10, seed=72), dev).view(1, 10, 33)
    rows = ids[0, -6:].clone()
    with torch.inference_mode():
        # eager: every piece of the reference's step run without graphs
        fast.prefill(ids)
        L0 = fast.m.seq_len
        eager = []
        for t in range(rows.shape[0]):
            fast.ids_row.copy_(rows[t].view(1, 33))
            fast.pos_dev.fill_(L0 + t)
            fast._run_eager(L0 + t + 1)
            eager.append((fast.lt_static.clone(), fast.la_static.clone(), fast.h_final.clone()))
        # graph replay from the same prefill
        fast.prefill(ids)
        fast.capture()
        base.prefill(ids)
        base.capture()
        for t in range(rows.shape[0]):
            lt, la, h, _ = fast.step(rows[t].view(1, 33), L0 + t)
            for a, b in zip(eager[t], (lt, la, h)):
                assert torch.equal(a.view(torch.int16), b.view(torch.int16)), t
            lt_b, la_b, h_b, _ = base.step(rows[t].view(1, 33), L0 + t)
            rel = float((h.float() - h_b.float()).norm() / h_b.float().norm())
            assert rel < 2e-2, (t, rel)
            assert (la.float().argmax(-1) == la_b.float().argmax(-1)).float().mean() > 0.85
