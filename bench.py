"""Benchmark: W4 decode steps/s at batch 1 under CUDA graph (config 2 of the
benchmark: 36 layers, hidden 4096, 32/8 heads, head_dim 128, SwiGLU 12288,
vocab 151936 + 32 x 1025 audio codebooks, RTN W4 g128, 128-row prompt).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mtl|reference]

One process per GPU (torchrun for N > 1); every GPU runs an independent
replica on its own utterance (no collective on the data path), so scaling is
weak and the value is the whole-job steps/s.

* ``value``  - K steps of the device-resident greedy decode loop: one CUDA
  graph per step (the whole decoder step in the audio phase plus a kernel
  that feeds the argmax tokens back as the next row), replayed back to back;
  weights (~3.9 GB per step) stream from HBM (inputs >> L2).
* ``e2e``    - the same metric through the public API ``generate_fast``
  (greedy): per step the graph replay, device-side decisions, a device->host
  read of the 33 tokens, the host FSM and a host->device copy of the next row.
* ``roofline`` - the dominant kernel (W4 GEMV): one graph of the 144 W4
  GEMV launches of a step (same weights, same launch order) timed with CUDA
  events; achieved = algorithmic bytes / average launch time.
* ``cpu_baseline`` / ``--impl reference`` - the numpy oracle (the CPU
  restatement of the reference decoder) timed on the host cores on a bounded
  sample of the same step, scaled to the full model.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(hidden=4096, n_layers=36, n_heads=32, n_kv=8, head_dim=128, inter=12288, vocab=151936,
           group_size=128, prompt_len=128, std=0.02, seed=0)
METRIC = "W4 decode steps/s at batch 1 (CUDA graph)"
MAX_SEQ = 8192


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _ncu_traffic():
    """Per-launch DRAM bytes of the W4 GEMV from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "w4_gemv_traffic.json")) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = f"/tmp/mtl_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ model
def synth_weights(dev, seed: int) -> dict:
    """Seeded random-init checkpoint of the configuration-2 model under the
    reference key names (model.py:55-105): the seven linears of every layer,
    the text embedding / head and the 32 audio embeddings / heads ~ N(0, 0.02)
    in bf16, norm weights 1."""
    import torch
    from moss_tts_lite_b200.model import N_VQ
    c = CFG
    H, D = c["hidden"], c["head_dim"]
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def r(*shape):
        return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * c["std"]).to(torch.bfloat16)

    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
    w = {"language_model.embed_tokens.weight": r(c["vocab"], H), "language_model.norm.weight": ones(H)}
    for li in range(c["n_layers"]):
        p = f"language_model.layers.{li}"
        w[f"{p}.input_layernorm.weight"] = ones(H)
        w[f"{p}.post_attention_layernorm.weight"] = ones(H)
        w[f"{p}.self_attn.q_proj.weight"] = r(c["n_heads"] * D, H)
        w[f"{p}.self_attn.k_proj.weight"] = r(c["n_kv"] * D, H)
        w[f"{p}.self_attn.v_proj.weight"] = r(c["n_kv"] * D, H)
        w[f"{p}.self_attn.o_proj.weight"] = r(H, c["n_heads"] * D)
        w[f"{p}.self_attn.q_norm.weight"] = ones(D)
        w[f"{p}.self_attn.k_norm.weight"] = ones(D)
        w[f"{p}.mlp.gate_proj.weight"] = r(c["inter"], H)
        w[f"{p}.mlp.up_proj.weight"] = r(c["inter"], H)
        w[f"{p}.mlp.down_proj.weight"] = r(H, c["inter"])
    for i in range(N_VQ):
        w[f"emb_ext.{i}.weight"] = r(1025, H)
    w["lm_heads.0.weight"] = r(c["vocab"], H)
    for i in range(N_VQ):
        w[f"lm_heads.{i + 1}.weight"] = r(1025, H)
    return w


def build_fast(dev, seed: int, max_seq: int = None):
    """Random-init (seeded) full-size synthetic model -> FastMossTTS(quant='w4')."""
    import torch
    from moss_tts_lite_b200.fast import FastMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    w = synth_weights(dev, seed)
    model = MossTTSModel(w, device=dev, max_seq_len=max_seq or MAX_SEQ)
    del w
    fast = FastMossTTS(model, quant="w4", w4_group_size=CFG["group_size"])
    torch.cuda.synchronize()
    return fast


def make_prompt(seed: int):
    import torch
    from moss_tts_lite_b200.model import AUDIO_START_TOKEN_ID, N_VQ
    g = torch.Generator().manual_seed(seed)
    L = CFG["prompt_len"]
    ids = torch.zeros(1, L, N_VQ + 1, dtype=torch.long)
    ids[0, :, 0] = torch.randint(0, 151643, (L,), generator=g)
    ids[0, :, 1:] = torch.randint(0, 1024, (L, N_VQ), generator=g)
    ids[0, -1, 0] = AUDIO_START_TOKEN_ID
    return ids


# --------------------------------------------------------------- measures
def time_decode_loop(fast, steps: int, warmup: int, dist_ctx):
    """Device-resident greedy decode: `steps` graph replays, CUDA-event timed."""
    import torch
    loop = fast.capture_greedy_loop()
    # continue the utterance after the prompt: capture() parked pos_dev on the
    # scratch slot, the feed kernel advances it from here on
    fast.pos_dev.fill_(CFG["prompt_len"])
    for _ in range(warmup):
        loop.replay()
    torch.cuda.synchronize()
    dist_ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(torch.cuda.current_device())
    with clocks:
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("mtl_timed")   # ncu --nvtx-include mtl_timed/ selects this region
        e0.record()
        for _ in range(steps):
            loop.replay()
        e1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    dist_ctx.barrier()
    return e0.elapsed_time(e1), clocks.summary()


def time_w4_gemvs(fast, reps: int = 5):
    """Roofline of the dominant kernel: the 144 W4 GEMV launches of one step
    in one graph (production order, same buffers and weights)."""
    import torch
    eng = fast.engine
    m = fast.m
    launches, alg = 0, 0

    def body():
        nonlocal launches, alg
        launches, alg = 0, 0
        for li in range(m.n_layers):
            lyr, L = m.layers[li], eng.lins[li]
            L["qkv"](eng.h, eng.qkv, norm_weight=lyr["input_layernorm"])
            L["o"](eng.attn, eng.h, residual=eng.h)
            L["gu"](eng.h, eng.act, norm_weight=lyr["post_attention_layernorm"], swiglu=True)
            L["down"](eng.act, eng.h, residual=eng.h)
            for name, res in (("qkv", 0), ("o", 1), ("gu", 0), ("down", 1)):
                w = L[name].w
                nout = w.N // 2 if name == "gu" else w.N
                alg += w.tiles.numel() + 2 * w.K + 2 * nout + (2 * w.N if res else 0)
                launches += 1

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    per_launch_s = ms * 1e-3 / launches
    per_launch_bytes = alg / launches
    return per_launch_bytes, per_launch_s, launches


def time_e2e(fast, prompt, steps: int, warmup: int):
    """generate_fast (public API, greedy) wall-clock steps/s over steps warmup..warmup+steps."""
    from moss_tts_lite_b200.fast import generate_fast
    st = {}
    res = generate_fast(fast, {"input_ids": prompt}, max_new_tokens=warmup + steps + 1, greedy=True,
                        watchdog=False, stats=st)
    wall = st.get("step_wall_s", [])
    n = min(len(wall) - 1, warmup + steps)
    if n <= warmup:
        return None, res.n_steps, st.get("relaunches")
    return (n - warmup) / (wall[n] - wall[warmup]), res.n_steps, st.get("relaunches")


def time_cfg3(fast, prompt_len: int = 4096, steps: int = 1024, seed: int = 3):
    """Configuration 3 through the public API: a 4096-row prompt (seeded random
    ids, last row AUDIO_START) prefilled, then `steps` sampled steps with
    audio temperature 0.8, top-k 50, top-p 0.95 (text at the reference
    defaults), watchdog off.  Cache lengths 4097..4096+steps."""
    import torch
    from moss_tts_lite_b200.fast import generate_fast
    from moss_tts_lite_b200.model import AUDIO_START_TOKEN_ID, N_VQ
    g = torch.Generator().manual_seed(seed)
    ids = torch.zeros(1, prompt_len, N_VQ + 1, dtype=torch.long)
    ids[0, :, 0] = torch.randint(0, 151643, (prompt_len,), generator=g)
    ids[0, :, 1:] = torch.randint(0, 1024, (prompt_len, N_VQ), generator=g)
    ids[0, -1, 0] = AUDIO_START_TOKEN_ID
    # one untimed prefill of the same length first: the first call in a
    # process also loads and selects the library GEMM / attention kernels
    fast.prefill(ids.to(fast.m.device))
    torch.cuda.synchronize()
    st = {}
    t0 = time.perf_counter()
    res = generate_fast(fast, {"input_ids": ids}, max_new_tokens=steps, seed=seed, audio_temperature=0.8,
                        audio_top_k=50, audio_top_p=0.95, watchdog=False, stats=st)
    t1 = time.perf_counter()
    wall = st.get("step_wall_s", [])
    n = len(wall)
    e2e = (n - 1) / (wall[-1] - wall[0]) if n > 1 else None
    dev = st.get("step_ms", [])
    phase = st.get("audio_phase", [])
    return {"workload": f"cfg3: {prompt_len}-row prompt, {n} sampled steps (audio T=0.8, top-k 50, top-p 0.95), "
                        f"cache {prompt_len + 1}..{prompt_len + n}",
            "e2e_steps_per_s": e2e, "device_ms_per_step_median": (statistics.median(dev) if dev else None),
            "audio_phase_frac": (sum(phase) / len(phase) if phase else None), "steps": res.n_steps,
            "prefill_s": (st.get("prefill_ms") or 0.0) / 1e3, "prefill_note": "after one untimed prefill call",
            "wall_s": t1 - t0,
            # audio-phase step bytes: weights + heads (3,883,599,872 B) + 147,456 B of K/V per cached position
            "roofline_ms_per_step_at_mean_cache": (3883599872 + 147456 * (prompt_len + n / 2)) / (_peaks()[0] * 1e6)}


def time_cfg4(fast, streams: int = 16, prompt_len: int = 256, steps: int = 2048, seed: int = 4):
    """Configuration 4: ``streams`` independent utterances per GPU, each a
    seeded random ``prompt_len``-row prompt (last row AUDIO_START) prefilled
    into its own KV cache, then ``steps`` batched greedy audio-phase decode
    steps replayed as one CUDA graph per step (every stream advances each
    step).  Device time by CUDA events; frames/s = streams x steps/s."""
    import torch
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    from moss_tts_lite_b200.model import AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_START_TOKEN_ID, N_VQ
    g = torch.Generator().manual_seed(seed)
    dev = fast.m.device
    bt = BatchedFastMossTTS(fast, streams, max_seq=prompt_len + steps + 8)
    t0 = time.perf_counter()
    for s in range(streams):
        ids = torch.zeros(prompt_len, N_VQ + 1, dtype=torch.long)
        ids[:, 0] = torch.randint(0, 151643, (prompt_len,), generator=g)
        ids[:, 1:] = torch.randint(0, 1024, (prompt_len, N_VQ), generator=g)
        ids[-1, 0] = AUDIO_START_TOKEN_ID
        bt.prefill(s, ids.to(dev))
        first = torch.cat([torch.tensor([AUDIO_GEN_SLOT_TOKEN_ID]), torch.randint(0, 1024, (N_VQ,), generator=g)])
        bt.start(s, first.to(dev), prompt_len)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    bt.capture()
    for _ in range(3):      # warm-up steps advance the streams like timed ones
        bt.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = steps - 3
    e0.record()
    for _ in range(n):
        bt.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    out = {"workload": f"cfg4: {streams} streams x {prompt_len}-row prompts (chunked W4 prefill per stream), "
                       f"{steps} batched greedy audio-phase steps, one graph per step",
           "streams": streams, "steps": steps, "device_ms_per_step": ms, "steps_per_s": 1e3 / ms,
           "frames_per_s": streams * 1e3 / ms, "prefill_s": prefill_s,
           "cache": f"{prompt_len + 1}..{prompt_len + steps} per stream"}
    del bt
    torch.cuda.empty_cache()
    return out


class CpuStep:
    """The numpy oracle decode step on the host cores, bounded sample: 2 of
    the 36 layers at the cfg2 shapes (fp32 BLAS on precomputed effective
    weights, KV length 129) plus embedding and audio-phase heads; one
    sample() times them once and scales the layers to the full model."""

    NL = 2

    def __init__(self):
        import numpy as np
        from oracle import step as ost
        from oracle.bf16 import f32_to_bf16
        c = CFG
        H, D = c["hidden"], c["head_dim"]
        rng = np.random.default_rng(1)

        def r(*shape):
            return f32_to_bf16((rng.standard_normal(shape, dtype=np.float32) * np.float32(c["std"])))

        w = {"language_model.embed_tokens.weight": np.zeros((c["vocab"], H), np.uint16),
             "language_model.norm.weight": f32_to_bf16(np.ones(H, np.float32))}
        for li in range(self.NL):
            p = f"language_model.layers.{li}"
            w[f"{p}.input_layernorm.weight"] = f32_to_bf16(np.ones(H, np.float32))
            w[f"{p}.post_attention_layernorm.weight"] = f32_to_bf16(np.ones(H, np.float32))
            w[f"{p}.self_attn.q_proj.weight"] = r(c["n_heads"] * D, H)
            w[f"{p}.self_attn.k_proj.weight"] = r(c["n_kv"] * D, H)
            w[f"{p}.self_attn.v_proj.weight"] = r(c["n_kv"] * D, H)
            w[f"{p}.self_attn.o_proj.weight"] = r(H, c["n_heads"] * D)
            w[f"{p}.self_attn.q_norm.weight"] = f32_to_bf16(np.ones(D, np.float32))
            w[f"{p}.self_attn.k_norm.weight"] = f32_to_bf16(np.ones(D, np.float32))
            w[f"{p}.mlp.gate_proj.weight"] = r(c["inter"], H)
            w[f"{p}.mlp.up_proj.weight"] = r(c["inter"], H)
            w[f"{p}.mlp.down_proj.weight"] = r(H, c["inter"])
        for i in range(32):
            w[f"emb_ext.{i}.weight"] = r(1025, H)
        w["lm_heads.0.weight"] = np.zeros((c["vocab"], H), np.uint16)
        for i in range(32):
            w[f"lm_heads.{i + 1}.weight"] = r(1025, H)
        self.ost = ost
        self.om = ost.OracleModel(w, max_seq_len=c["prompt_len"] + 8, fp32_linears=True)
        self.om.seq = c["prompt_len"]
        self.row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
        try:
            from threadpoolctl import threadpool_info
            self.cores = max(int(i.get("num_threads", 1)) for i in threadpool_info()) or (os.cpu_count() or 1)
        except Exception:
            self.cores = os.cpu_count() or 1
        self.sample_desc = (f"numpy oracle step at cfg2 shapes: {self.NL} of {CFG['n_layers']} layers timed (fp32 "
                            f"BLAS, effective weights precomputed, KV length {CFG['prompt_len'] + 1}) + embedding + "
                            f"audio-phase heads per sample, layers scaled to {CFG['n_layers']}")

    def sample(self) -> float:
        """Seconds of one full decode step (estimated from this sample)."""
        om, ost = self.om, self.ost
        t0 = time.perf_counter()
        h = om.embed_rows(self.row.reshape(1, -1))
        t1 = time.perf_counter()
        for li in range(self.NL):
            h = om.layer(li, h, om.seq)
        t2 = time.perf_counter()
        hf = ost.rms_norm(h, om.final_norm)
        om.text_logits_2way(hf)
        om.audio_logits(hf)
        t3 = time.perf_counter()
        return (t1 - t0) + (t3 - t2) + (t2 - t1) * CFG["n_layers"] / self.NL


def cpu_baseline(reps: int = 3):
    """(steps/s, cores, sample description) of the CPU oracle step."""
    cs = CpuStep()
    cs.sample()  # warm
    per_step = statistics.median(cs.sample() for _ in range(reps))
    return 1.0 / per_step, cs.cores, cs.sample_desc + f", median of {reps} samples"


# ------------------------------------------------------------------- main
class _Dist:
    """One process per GPU (torchrun env): the replicas share nothing on the
    data path; the process group only aligns the timed regions (barrier) and
    takes the max over ranks of the device times.  NCCL on the GPU box; gloo
    (host tensors) for the CPU tests of this logic."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        self.device = "cuda"

    def init(self, backend: str = "nccl"):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            import torch
            kw = {"device_id": torch.device("cuda", self.local)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.pg = dist
            self.device = "cuda" if backend == "nccl" else "cpu"

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if self.pg is None:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def run_reference_arm(args, ctx):
    """--impl reference: the CPU restatement of the reference path (numpy
    oracle) on the host cores; rank 0 only.  Each step is one bounded sample
    of the decode step (CpuStep.sample), so K steps take K x ~0.5 s."""
    if ctx.rank != 0:
        return
    cs = CpuStep()
    for _ in range(max(1, args.warmup)):
        cs.sample()
    vals = [1.0 / cs.sample() for _ in range(args.steps)]
    cores, sample = cs.cores, cs.sample_desc
    v = statistics.median(vals)
    line = {"metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg2: full synthetic MOSS-TTS-shaped W4 decode step, batch 1",
                       "model": "synthetic MOSS-TTS (36L, h4096, 32/8 heads, ffn 12288)"},
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_gemv(launches: int = 6):
    """Small case for ncu: config 0 (AutoGPTQ W4 linear 4096 -> 12288, g128,
    seeded synthetic tensors) on cuda:0, `launches` launches over 4 weight
    copies (105 MB, > L2)."""
    import numpy as np
    import torch
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import QuantLinear
    from oracle import w4 as ow
    dev = torch.device("cuda", 0)
    K, N, g = 4096, 12288, 128
    d = ow.synth_gptq_linear(K, N, g, seed=0)

    def t(a, dtype=None):
        x = torch.from_numpy(np.ascontiguousarray(a))
        return (x.view(dtype) if dtype is not None else x).to(dev)
    lins = [QuantLinear.from_tensors(t(d["qweight"]), t(d["qzeros"]), t(d["scales"], torch.float16),
                                     t(d["g_idx"]), group_size=g) for _ in range(4)]
    x = t(d["x"], torch.bfloat16)
    out = torch.empty(1, N, dtype=torch.bfloat16, device=dev)
    for i in range(launches):
        lins[i % 4].w.linear(x, out=out)
    torch.cuda.synchronize()
    st = _lib.device_status()
    print(json.dumps({"profile": "w4_gemv cfg0", "launches": launches, "bytes_per_launch": lins[0].w.tiles.numel()
                      + 2 * K + 2 * N, "device_status": st}))
    if st != 0:
        raise SystemExit(1)


def profile_heads(launches: int = 3):
    """Small case for ncu: the text-phase head of configuration 2 alone, the
    final RMSNorm fused into the bf16 GEMV over the [151936, 4096] text head
    (1.245 GB, > L2; seeded synthetic weights), `launches` launches."""
    import torch
    from moss_tts_lite_b200 import _lib, kernels
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    H, V = CFG["hidden"], CFG["vocab"]
    W = (torch.randn(V, H, generator=g, device=dev) * CFG["std"]).to(torch.bfloat16)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    h = torch.randn(1, H, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(1, V, dtype=torch.bfloat16, device=dev)
    hn = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    for _ in range(launches):
        kernels.bf16_linear(h, W, out, norm_weight=nw, eps=1e-6, x_normed=hn)
    torch.cuda.synchronize()
    st = _lib.device_status()
    print(json.dumps({"profile": "bf16_gemv text head", "launches": launches, "bytes_per_launch": V * H * 2 + 4 * H
                      + 2 * V, "device_status": st}))
    if st != 0:
        raise SystemExit(1)


def profile_cfg4(steps: int = 2):
    """Configuration 4's batched step (16 streams, 256-row prompts) with
    `steps` graph replays inside the NVTX range `mtl_timed` (the ncu launch-
    list case)."""
    import torch
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    from moss_tts_lite_b200.model import AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_START_TOKEN_ID, N_VQ
    dev = torch.device("cuda", 0)
    fast = build_fast(dev, seed=CFG["seed"])
    g = torch.Generator().manual_seed(4)
    bt = BatchedFastMossTTS(fast, 16, max_seq=512)
    for s in range(16):
        ids = torch.zeros(256, N_VQ + 1, dtype=torch.long)
        ids[:, 0] = torch.randint(0, 151643, (256,), generator=g)
        ids[:, 1:] = torch.randint(0, 1024, (256, N_VQ), generator=g)
        ids[-1, 0] = AUDIO_START_TOKEN_ID
        bt.prefill(s, ids.to(dev))
        first = torch.cat([torch.tensor([AUDIO_GEN_SLOT_TOKEN_ID]), torch.randint(0, 1024, (N_VQ,), generator=g)])
        bt.start(s, first.to(dev), 256)
    bt.capture()
    for _ in range(3):
        bt.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("mtl_timed")
    for _ in range(steps):
        bt.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"profile": "cfg4 batched step", "steps": steps}))


def profile_attn(timed: bool = True, launches: int = 4, lengths=(136, 1024, 4096, 8191)):
    """Decode attention of configuration 2 alone (32 query / 8 KV heads x 128,
    KV cache [8, 8192, 128] for one layer, seeded synthetic values): per cache
    length, the device time of 50 launches chained in a CUDA graph (if
    `timed`), then `launches` plain launches at the first length (the ncu
    capture case)."""
    import torch
    from moss_tts_lite_b200 import _lib, kernels
    from moss_tts_lite_b200.model import rope_tables
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    nh, nkv, hd, max_seq = CFG["n_heads"], CFG["n_kv"], CFG["head_dim"], MAX_SEQ
    splits = 16

    def r(*shape, s=1.0):
        return (torch.randn(*shape, generator=g) * s).to(torch.bfloat16).to(dev)
    qkv = r(1, (nh + 2 * nkv) * hd)
    qn, kn = r(hd, s=0.1) + 1, r(hd, s=0.1) + 1
    cos, sin = rope_tables(max_seq, dev, torch.bfloat16, hd)
    kc, vc = r(nkv, max_seq, hd), r(nkv, max_seq, hd)
    out = torch.empty(1, nh * hd, dtype=torch.bfloat16, device=dev)
    scratch = torch.zeros(_lib.attn_scratch_bytes(1, nh, nkv, splits), dtype=torch.uint8, device=dev)
    pos = torch.zeros(1, dtype=torch.int64, device=dev)

    def launch(stable=False):
        kernels.attn_decode(qkv, qn, kn, cos, sin, kc, vc, pos, nh, nkv, splits, out, scratch, kv_stable=stable)
    res = {}
    s = torch.cuda.Stream(device=dev)
    for L in (lengths if timed else ()):
        pos.fill_(L - 1)
        with torch.cuda.stream(s):
            launch()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                for _ in range(50):
                    launch(stable=True)
            for _ in range(3):
                gr.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(10):
                gr.replay()
            e1.record(s)
            e1.synchronize()
            res[L] = e0.elapsed_time(e1) * 1e3 / 500
            del gr
    pos.fill_(lengths[0] - 1)
    for _ in range(launches):
        launch()
    torch.cuda.synchronize()
    st = _lib.device_status()
    print(json.dumps({"profile": "attn_decode cfg2", "us_per_launch_in_graph": res, "launches": launches,
                      "device_status": st}))
    if st != 0:
        raise SystemExit(1)


def run_reference_gpu(args, ctx):
    """--impl reference-gpu (informational, rank 0): the unmodified reference
    W4 fast path on this GPU through its public API - moss_tts_lite.model.
    MossTTSModel + moss_tts_lite.fast.FastMossTTS(quant='w4', g128, tinygemm)
    + generate_fast(greedy) - on the same synthetic model and prompt; decode
    steps/s from generate_fast's own per-step CUDA-event stats, skipping the
    warm-up steps.  Needs the reference package under baseline/_ref."""
    import torch
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if ref_dir not in sys.path:
        sys.path.append(ref_dir)
    try:
        from moss_tts_lite.fast import FastMossTTS as RefFast
        from moss_tts_lite.fast import generate_fast as ref_generate_fast
        from moss_tts_lite.model import MossTTSModel as RefModel
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"reference package not importable: {e}"}))
        return
    if ctx.rank != 0:
        return
    dev = torch.device("cuda", ctx.local)
    torch.cuda.set_device(dev)
    c = CFG
    w = synth_weights(dev, c["seed"])
    model = RefModel(w, device=dev, dtype=torch.bfloat16, max_seq_len=MAX_SEQ)
    del w
    fast = RefFast(model, quant="w4", w4_group_size=c["group_size"])
    prompt = make_prompt(c["seed"]).to(dev)
    st = {}
    n = args.warmup + args.steps + 1
    res = ref_generate_fast(fast, {"input_ids": prompt}, max_new_tokens=n, greedy=True, watchdog=False, stats=st)
    ms = st["step_ms"][args.warmup:args.warmup + args.steps]
    v = 1000.0 / (sum(ms) / len(ms))
    print(json.dumps({"metric": METRIC, "impl": "reference-gpu", "value": v, "unit": "steps/s",
                      "ms_per_step": 1000.0 / v, "steps": len(ms), "warmup": args.warmup,
                      "steps_generated": res.n_steps,
                      "what": "moss_tts_lite FastMossTTS(quant='w4', g128) + generate_fast(greedy), same "
                              "synthetic model and prompt, per-step CUDA-event stats of the reference"}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="mtl", choices=["mtl", "reference", "reference-gpu"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cfg3", action="store_true", help="skip the long-context sampled configuration-3 run")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the 16-stream batched configuration-4 run")
    ap.add_argument("--profile-gemv", action="store_true", help="small config-0 GEMV case for ncu")
    ap.add_argument("--profile-attn", action="store_true", help="decode attention alone (config 2 heads)")
    ap.add_argument("--profile-attn-launches", action="store_true", help="4 plain attention launches (ncu case)")
    ap.add_argument("--attn-len", type=int, default=136, help="cache length of the plain attention launches")
    ap.add_argument("--profile-heads", action="store_true", help="text-head bf16 GEMV alone (ncu case)")
    ap.add_argument("--profile-cfg4", action="store_true", help="2 batched configuration-4 steps in an NVTX range")
    args = ap.parse_args()
    if args.profile_heads:
        profile_heads()
        return
    if args.profile_cfg4:
        profile_cfg4()
        return
    if args.profile_gemv:
        profile_gemv()
        return
    if args.profile_attn or args.profile_attn_launches:
        lengths = (args.attn_len,) + tuple(L for L in (136, 1024, 4096, 8191) if L != args.attn_len)
        profile_attn(timed=args.profile_attn, lengths=lengths)
        return
    ctx = _Dist()
    if ctx.world > 1 and args.gpus != ctx.world:
        raise SystemExit(f"--gpus {args.gpus} does not match the {ctx.world} ranks torchrun started")
    if args.impl == "reference":
        run_reference_arm(args, ctx)
        return
    if args.impl == "reference-gpu":
        run_reference_gpu(args, ctx)
        return
    import torch
    torch.cuda.set_device(ctx.local)
    ctx.init()
    dev = torch.device("cuda", ctx.local)
    t_build = time.time()
    fast = build_fast(dev, seed=CFG["seed"] + ctx.rank)
    prompt = make_prompt(CFG["seed"] + ctx.rank)
    fast.prefill(prompt.to(dev))
    fast.capture()
    build_s = time.time() - t_build
    steps, warmup = args.steps, max(3, args.warmup)
    ms, clocks = time_decode_loop(fast, steps, warmup, ctx)
    ms = ctx.max(ms)
    ms_per_step = ms / steps
    value = ctx.world * steps / (ms * 1e-3)
    bytes_per_launch, s_per_launch, launches = time_w4_gemvs(fast)
    e2e, e2e_steps, e2e_relaunches = time_e2e(fast, prompt.to("cpu"), steps, warmup)
    e2e_all = ctx.max(-(e2e or 0.0))  # slowest rank
    e2e_val = ctx.world * (-e2e_all) if e2e else None
    peak, peak_kind = _peaks()
    achieved = bytes_per_launch / s_per_launch / 1e9
    traffic = _ncu_traffic()
    cfg3 = None
    if ctx.rank == 0 and args.gpus == 1 and not args.no_cfg3:
        cfg3 = time_cfg3(fast)
    cfg4 = None
    if ctx.rank == 0 and args.gpus == 1 and not args.no_cfg4:
        cfg4 = time_cfg4(fast)
    cpu = None
    if ctx.rank == 0 and args.gpus == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_baseline()
        cpu = {"value": v, "unit": "steps/s", "cores": cores, "kind": "port", "sample": sample}
    if ctx.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2: full synthetic MOSS-TTS-shaped W4 decode step, batch 1",
                       "model": "synthetic MOSS-TTS (36L, h4096, 32/8 heads x128, ffn 12288, vocab 151936 + "
                                "32x1025 codebooks, RTN W4 g128, random-init seed 0)",
                       "global_batch": args.gpus, "seq_len": CFG["prompt_len"], "parallelism": f"replicas{args.gpus}",
                       "phase": "audio (2-way text head + 32 audio heads), greedy tokens fed back on device",
                       "l2": "inputs larger than L2 (~3.9 GB of weights per step)",
                       "weights": "int4 codes + bf16 (scale, zero) per 128-group; activations bf16, fp32 accumulate",
                       "build_s": round(build_s, 1)},
            # per step: the 33 decisions come back to the host (pinned, 264 B);
            # the next input row is built on the device from them (as the
            # reference builds current_input_ids), so no per-step h2d copy;
            # the prompt crosses once per call
            "e2e": {"value": e2e_val, "unit": "steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 33 * 8, "h2d_prompt_bytes": int(prompt.numel()) * 8,
                    "api": "moss_tts_lite_b200.fast.generate_fast(greedy=True)",
                    "steps_generated": e2e_steps, "speculation_relaunches": e2e_relaunches},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         # ncu DRAM bytes of the config-0 capture, scaled by its
                         # traffic/algorithmic ratio to the average step launch
                         "traffic": (bytes_per_launch * traffic["traffic_over_algorithmic"]
                                     if traffic else None),
                         "kernel": "w4_gemv_kernel (144 launches per step: q|k|v, o, gate|up, down x 36)",
                         "bytes_per_launch": bytes_per_launch, "us_per_launch": s_per_launch * 1e6},
            "gpu_launches": steps * (1 + 5 * CFG["n_layers"] + 2 + 1),
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if cfg3 is not None:
            line["cfg3"] = cfg3
        if cfg4 is not None:
            line["cfg4"] = cfg4
        print(json.dumps(line), flush=True)
    ctx.barrier()
    del fast
    ctx.close()


if __name__ == "__main__":
    main()
