"""``synthesize()`` (moss_tts_lite/cli.py:287-322) with the decode on the B200 kernels.

The stages around the decode are not part of this package: the text front
end (``build_tts_prompt``), the safetensors loader and the audio codec are
taken from the reference package, which must be importable (with
``soundfile`` for the wav file).  What runs here is the decode itself:
``FastMossTTS`` (``quant`` None = bf16 or "w4" = RTN W4) or, with
``gptq_state``, ``GptqMossTTS`` from ``load_gptq_fast``, driven by this
package's ``generate_fast``.  Same keyword arguments and return value as
the reference: ``(wav, sample_rate, GenResult, strategy)``, where strategy
is "resident" (codec loaded next to the decoder) or "sequential" (decoder
freed before the codec, after an out-of-memory error).

Not served: standalone quantized exports as ``model_dir`` (their loader is
not built here), ``fast=False`` (the reference's eager loop) and
``fast_native`` (the reference's n2 arm: this package's decode already runs
one graph per step on the device).
"""
from __future__ import annotations

import sys

import numpy as np
import torch

from .fast import FastMossTTS, generate_fast
from .gptq import load_gptq_fast


def _reference_cli():
    try:
        from moss_tts_lite import cli
    except ImportError as e:
        raise ImportError("synthesize() takes the text front end, the weight loader and the codec from the "
                          "reference package moss_tts_lite (with soundfile), which is not importable: "
                          f"{e}") from e
    return cli


def _decode(rc, text, *, dev, language, seed, greedy, max_new_tokens, model_dir, quant, w4_group_size, gptq_state,
            max_seq_len, sampling, watchdog, watchdog_silence_frames, watchdog_max_segment_frames, stats):
    """Prompt -> decoder -> generate_fast; returns (GenResult, decode stats)."""
    prompt = rc.build_tts_prompt(text, language=language, tokenizer=None)
    l0 = int(prompt["input_ids"].shape[1])
    positions = max(l0 + max_new_tokens + rc.KV_RAMP_MARGIN, int(max_seq_len or 0))
    model = rc._load_tts(model_dir, dev, positions)
    try:
        if gptq_state:
            decoder = load_gptq_fast(model, gptq_state)
        else:
            kw = {} if w4_group_size is None else {"w4_group_size": w4_group_size}
            decoder = FastMossTTS(model, quant=quant, **kw)
        res = generate_fast(decoder, prompt, max_new_tokens=max_new_tokens, seed=seed, greedy=greedy,
                            watchdog=watchdog, watchdog_silence_frames=watchdog_silence_frames,
                            watchdog_max_segment_frames=watchdog_max_segment_frames,
                            max_requested_pause_s=rc._max_pause_s(text), stats=stats, **sampling)
        info = {"max_seq_len": int(model.max_seq_len), "l0": l0}
        del decoder
    finally:
        del model
        torch.cuda.empty_cache()
    return res, info


def synthesize(text: str, output: str, *, language=None, seed=1234, greedy=False, max_new_tokens=4096,
               device="cuda", model_dir=None, codec_dir=None, chunk_duration=8.0, sampling: dict | None = None,
               stats: dict | None = None, fast=True, quant=None, w4_group_size=None, watchdog=True,
               watchdog_silence_frames=None, watchdog_max_segment_frames=None, gptq_state=None, fast_native=False,
               max_seq_len=None, max_graphs=None):
    """End-to-end text -> wav, the decode on this package's kernels."""
    rc = _reference_cli()
    if not fast:
        raise ValueError("synthesize(fast=False) is the reference's eager loop; this package serves the graph decode")
    if fast_native:
        raise ValueError("synthesize(fast_native=True) is the reference's n2 arm; this package's graph decode "
                         "already runs each step as one graph")
    model_dir = model_dir or rc.MODEL_DIR
    codec_dir = codec_dir or rc.CODEC_DIR
    if rc.is_standalone_dir(model_dir):
        raise NotImplementedError(f"{model_dir} is a standalone quantized export, whose loader is not built here")
    sampling = {k: v for k, v in (sampling or {}).items() if v is not None}
    dev = torch.device(device)
    tstats: dict = {}
    strategy = "resident"
    codec = None
    while True:
        try:
            if strategy == "resident":
                codec = rc.MossCodecDecoder(codec_dir, device=dev)
            res, info = _decode(rc, text, dev=dev, language=language, seed=seed, greedy=greedy,
                                max_new_tokens=max_new_tokens, model_dir=model_dir, quant=quant,
                                w4_group_size=w4_group_size, gptq_state=gptq_state, max_seq_len=max_seq_len,
                                sampling=sampling, watchdog=watchdog, watchdog_silence_frames=watchdog_silence_frames,
                                watchdog_max_segment_frames=watchdog_max_segment_frames, stats=tstats)
            break
        except torch.cuda.OutOfMemoryError:
            if strategy != "resident":
                raise
            print("[moss_tts_lite_b200] CUDA out of memory with the codec resident; retrying with the decoder "
                  "freed before the codec is loaded", file=sys.stderr)
            codec = None
            torch.cuda.empty_cache()
            strategy = "sequential"
    if codec is None:
        codec = rc.MossCodecDecoder(codec_dir, device=dev)
    segments = rc.delayed_rows_to_segments(res.audio_frames)
    pieces = [codec.decode(seg, chunk_duration=chunk_duration) for seg in segments]
    wav = pieces[0] if len(pieces) == 1 else np.concatenate(pieces)
    rc.sf.write(output, wav, rc.SR, subtype="FLOAT")
    tstats.update(info)
    if stats is not None:
        stats.update(tstats)
    return wav, rc.SR, res, strategy
