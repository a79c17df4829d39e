"""synthesize() (moss_tts_lite/cli.py:287-322) with the decode on this
package: the reference's text front end, loader and codec are replaced by
stubs (the real weights, tokenizer files and codec are not in this
environment; soundfile is stubbed too), and the decode must be this
package's generate_fast over its FastMossTTS, giving the tokens a direct
generate_fast call gives, with the reference's return value
(wav, sample rate, GenResult, strategy)."""
import sys
import types

import numpy as np
import pytest
import torch

from conftest import require_cuda
from test_step_gpu import _prompt, _t, _torch_weights, _weights

pytestmark = pytest.mark.gpu


def test_synthesize_runs_the_b200_decode(monkeypatch, tmp_path):
    dev = require_cuda()
    written = {}
    fake_sf = types.ModuleType("soundfile")
    fake_sf.write = lambda path, data, sr, subtype=None: written.update(path=path, n=len(data), sr=sr)
    monkeypatch.setitem(sys.modules, "soundfile", fake_sf)
    rcli = pytest.importorskip("moss_tts_lite.cli")
    ref_model = pytest.importorskip("moss_tts_lite.model")
    monkeypatch.setattr(rcli, "sf", fake_sf)
    w = _weights(seed=81)
    ids = _t(_prompt(12, seed=82), dev).view(1, 12, 33)

    class FakeCodec:
        def __init__(self, path, device=None):
            self.path = path

        def decode(self, seg, chunk_duration=8.0):
            return np.zeros(len(seg) * 1920, np.float32)

    monkeypatch.setattr(rcli, "MossCodecDecoder", FakeCodec)
    monkeypatch.setattr(rcli, "is_standalone_dir", lambda p: False)
    monkeypatch.setattr(rcli, "delayed_rows_to_segments", lambda frames: [frames])
    monkeypatch.setattr(rcli, "build_tts_prompt", lambda text, language=None, tokenizer=None:
                        {"input_ids": ids.cpu(), "attention_mask": torch.ones(1, 12, dtype=torch.bool)})
    monkeypatch.setattr(rcli, "_load_tts", lambda d, device, max_seq_len=8192: ref_model.MossTTSModel(
        _torch_weights(w, dev), device=device, dtype=torch.bfloat16, max_seq_len=max_seq_len))
    from moss_tts_lite_b200.cli import synthesize
    from moss_tts_lite_b200.fast import FastMossTTS, generate_fast
    from moss_tts_lite_b200.generate import GenResult
    stats = {}
    wav, sr, res, strategy = synthesize("hello", str(tmp_path / "out.wav"), greedy=True, max_new_tokens=24,
                                        quant="w4", model_dir="m", codec_dir="c", stats=stats)
    assert sr == 24000 and strategy == "resident" and isinstance(res, GenResult)
    assert written["path"] == str(tmp_path / "out.wav") and written["sr"] == 24000 and written["n"] == len(wav)
    assert stats["l0"] == 12 and res.n_steps >= 1
    direct = generate_fast(FastMossTTS(ref_model.MossTTSModel(_torch_weights(w, dev), device=dev, dtype=torch.bfloat16,
                                                              max_seq_len=stats["max_seq_len"]), quant="w4"),
                           {"input_ids": ids}, max_new_tokens=24, greedy=True)
    assert res.text_ids.tolist() == direct.text_ids.tolist()
    assert torch.equal(res.audio_frames, direct.audio_frames)
    with pytest.raises(ValueError):
        synthesize("hello", str(tmp_path / "x.wav"), fast=False, model_dir="m", codec_dir="c")
