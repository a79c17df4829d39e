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
* ``roofline`` - the dominant kernel: the persistent W4 chain (37 launches
  per step: o -> gate|up -> down -> next q|k|v per layer; the 144
  one-linear GEMV launches with MTL_CHAIN=0), in one graph with the same
  weights and launch order, timed with CUDA events; achieved = algorithmic
  bytes / average launch time.
* ``cpu_baseline`` / ``--impl reference`` - the reference's own decoder
  (MossTTSModel) on the host cores (the numpy oracle when the reference
  package is absent), on a bounded sample of the same step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(hidden=4096, n_layers=36, n_heads=32, n_kv=8, head_dim=128, inter=12288, vocab=151936,
           group_size=128, prompt_len=128, std=0.02, seed=0)
METRIC = "W4 decode steps/s at batch 1 (CUDA graph); int4 GEMV HBM GB/s vs B200 peak"
MAX_SEQ = 8192


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _ncu_traffic(name: str = "w4_gemv_traffic.json"):
    """DRAM traffic / algorithmic bytes of the W4 kernel from its committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 10 ms by a
    host thread through NVML while the timed region runs (reads only; no
    setting of the GPU is touched).  Falls back to `nvidia-smi -lms 200`
    when NVML is unavailable."""

    PERIOD_S = 0.01
    # NVML clocks-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.max_mhz = None
        self.err = None
        self._stop = None
        self._thread = None

    def _run(self):
        import pynvml
        h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                rs = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((sm, rs))
            except Exception as e:  # noqa: BLE001
                self.err = str(e)
            self._stop.wait(self.PERIOD_S)

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
            # NVML counts all GPUs; map the visible ordinal when it is numeric
            if idx and idx[0].strip().isdigit() and self.index < len(idx):
                self.index = int(idx[self.index])
        except Exception as e:  # noqa: BLE001
            self.err = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [self.err or "no samples"],
                    "samples": 0}
        reasons = sorted({name for _, rs in self.samples for bit, name in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(v for v, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "period_ms": self.PERIOD_S * 1e3,
                "source": "nvml"}


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
    """Roofline of the dominant kernel, timed as the step runs it: with the
    persistent chain (the default), its 37 launches of one step (q|k|v of
    layer 0, then o -> gate|up -> down -> next q|k|v per layer) in one graph;
    else the 144 W4 GEMV launches.  Production order, buffers and weights;
    algorithmic bytes = packed weights + x / y / residual rows."""
    import torch
    from moss_tts_lite_b200 import kernels
    from moss_tts_lite_b200.model import RMS_EPS
    eng = fast.engine
    m = fast.m
    launches, alg = 0, 0
    if eng.strips is not None:
        def phase_bytes(ph):
            w = ph["w"]
            nout = w.N // 2 if ph.get("swiglu") else w.N
            return w.tiles.numel() + 2 * w.K + 2 * nout + (2 * w.N if ph.get("residual") is not None else 0)

        def body():
            nonlocal launches, alg
            launches, alg = 0, 0
            seq = [[eng._phase(0, "qkv")]]
            for li in range(m.n_layers):
                ph = [eng._phase(li, nm) for nm in ("o", "gu", "down")]
                if li + 1 < m.n_layers:
                    ph.append(eng._phase(li + 1, "qkv"))
                seq.append(ph)
            for i, ph in enumerate(seq):
                kernels.w4_chain(ph, eng.chain_g, eng.chain_bar[i], RMS_EPS)
                alg += sum(phase_bytes(p) for p in ph)
                launches += 1
        return _graph_launch_time(body, reps, lambda: (alg, launches))

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

    return _graph_launch_time(body, reps, lambda: (alg, launches))


def _graph_launch_time(body, reps, totals):
    """(bytes per launch, seconds per launch, launches) of `body` replayed as
    one CUDA graph; `totals()` gives (algorithmic bytes, launches) of one body."""
    import torch
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
    alg, launches = totals()
    del g
    return alg / launches, ms * 1e-3 / launches, launches


def time_e2e(fast, prompt, steps: int, warmup: int):
    """generate_fast (public API, greedy) wall-clock steps/s over steps
    warmup..warmup+steps, and the phase mix of those steps (audio-phase steps
    run the 2-way head, text-phase steps the 1.245 GB text head)."""
    from moss_tts_lite_b200.fast import generate_fast
    st = {}
    res = generate_fast(fast, {"input_ids": prompt}, max_new_tokens=warmup + steps + 1, greedy=True,
                        watchdog=False, stats=st)
    wall = st.get("step_wall_s", [])
    n = min(len(wall) - 1, warmup + steps)
    phases = st.get("audio_phase", [])[warmup:n]
    mix = {"audio_phase_steps": int(sum(phases)), "text_phase_steps": int(len(phases) - sum(phases))}
    if n <= warmup:
        return None, res.n_steps, st.get("relaunches"), mix
    return (n - warmup) / (wall[n] - wall[warmup]), res.n_steps, st.get("relaunches"), mix


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
            "prefill_s": (st.get("prefill_ms") or 0.0) / 1e3,
            "prefill_note": "first prefill call at this prompt length (no warm-up call)",
            "wall_s": t1 - t0,
            # audio-phase step bytes: weights + heads (3,883,599,872 B) + 147,456 B of K/V per cached position
            "roofline_ms_per_step_at_mean_cache": (3883599872 + 147456 * (prompt_len + n / 2)) / (_peaks()[0] * 1e6)}


def time_cfg4(fast, streams: int = 16, prompt_len: int = 256, steps: int = 2048, seed: int = 4, tc: bool = False):
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
    bt = BatchedFastMossTTS(fast, streams, max_seq=prompt_len + steps + 8, tc=True if tc else None)
    prompts, firsts = [], []
    for s in range(streams):
        ids = torch.zeros(prompt_len, N_VQ + 1, dtype=torch.long)
        ids[:, 0] = torch.randint(0, 151643, (prompt_len,), generator=g)
        ids[:, 1:] = torch.randint(0, 1024, (prompt_len, N_VQ), generator=g)
        ids[-1, 0] = AUDIO_START_TOKEN_ID
        prompts.append(ids)
        firsts.append(torch.cat([torch.tensor([AUDIO_GEN_SLOT_TOKEN_ID]),
                                 torch.randint(0, 1024, (N_VQ,), generator=g)]))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    bt.prefill_all([p.to(dev) for p in prompts])        # all streams' rows in each GEMM (M = streams x L)
    for s in range(streams):
        bt.start(s, firsts[s].to(dev), prompt_len)
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
    out = {"workload": f"cfg4: {streams} streams x {prompt_len}-row prompts (prefilled together: tcgen05 W4 GEMMs "
                       f"over M = {streams} x {prompt_len} rows, causal GQA attention per stream), "
                       f"{steps} batched greedy audio-phase steps, one graph per step",
           "streams": streams, "steps": steps, "device_ms_per_step": ms, "steps_per_s": 1e3 / ms,
           "frames_per_s": streams * 1e3 / ms, "prefill_s": prefill_s,
           "prefill_note": "first call of the batched prefill in the process (host-timed, synchronised)",
           "cache": f"{prompt_len + 1}..{prompt_len + steps} per stream",
           "decode_linears": ("batched persistent chain (mtl_w4_chain_rows)" if bt.chain else
                              "tcgen05 tiles, one launch per linear (w4_tcb_kernel)" if bt.tc else
                              "register-MMA tiles, one launch per linear")}
    del bt
    torch.cuda.empty_cache()
    return out


def _host_threads() -> int:
    """Host cores this process may use (affinity), whatever OMP_NUM_THREADS
    torchrun set: the CPU baselines use all of them."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def _ref_package():
    """The unmodified reference package (a copy under baseline/_ref), or None."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(ref_dir) and ref_dir not in sys.path:
        sys.path.append(ref_dir)
    try:
        import moss_tts_lite.gptq  # noqa: F401
        import moss_tts_lite.model  # noqa: F401
        return sys.modules["moss_tts_lite"]
    except Exception:  # noqa: BLE001
        return None


class CpuRefStep:
    """The reference's own eager decoder on the host cores: moss_tts_lite.
    model.MossTTSModel (device='cpu', bf16) at the configuration-2 shapes, all
    36 layers, one audio-phase decode step = step(row) + text_logits_2way +
    audio_logits, starting at cache length 129.  bf16 random weights stand in
    for the dequantised effective weights (the reference's CPU W4 path runs
    them as bf16 F.linear); four distinct layer weight sets (1.5 GB) are
    cycled over the 36 layers to bound host memory, so every layer still
    streams its 386 MB of weights from DRAM (the set exceeds any LLC).  The
    K/V cache rows 0..127 are random (their values do not change the work)."""

    DISTINCT = 4

    def __init__(self, threads: int, steps: int):
        import torch
        ref = _ref_package()
        if ref is None:
            raise RuntimeError("reference package not importable")
        torch.set_num_threads(threads)
        self.cores = torch.get_num_threads()
        c = CFG
        H, D = c["hidden"], c["head_dim"]
        g = torch.Generator().manual_seed(1)

        def r(*shape):
            return (torch.randn(*shape, generator=g) * c["std"]).to(torch.bfloat16)
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16)  # noqa: E731
        sets = []
        for _ in range(self.DISTINCT):
            sets.append({"self_attn.q_proj.weight": r(c["n_heads"] * D, H), "self_attn.k_proj.weight": r(c["n_kv"] * D, H),
                         "self_attn.v_proj.weight": r(c["n_kv"] * D, H), "self_attn.o_proj.weight": r(H, c["n_heads"] * D),
                         "mlp.gate_proj.weight": r(c["inter"], H), "mlp.up_proj.weight": r(c["inter"], H),
                         "mlp.down_proj.weight": r(H, c["inter"])})
        w = {"language_model.embed_tokens.weight": r(c["vocab"], H), "language_model.norm.weight": ones(H)}
        for li in range(c["n_layers"]):
            p = f"language_model.layers.{li}"
            for k, t in sets[li % self.DISTINCT].items():
                w[f"{p}.{k}"] = t
            for k, n in (("input_layernorm", H), ("post_attention_layernorm", H), ("self_attn.q_norm", D),
                         ("self_attn.k_norm", D)):
                w[f"{p}.{k}.weight"] = ones(n)
        for i in range(32):
            w[f"emb_ext.{i}.weight"] = r(1025, H)
            w[f"lm_heads.{i + 1}.weight"] = r(1025, H)
        w["lm_heads.0.weight"] = r(c["vocab"], H)
        L = c["prompt_len"]
        self.m = ref.model.MossTTSModel(w, device="cpu", dtype=torch.bfloat16, max_seq_len=L + steps + 8)
        del w
        self.m.k_cache[:, :, :L].copy_(torch.randn(self.m.k_cache[:, :, :L].shape, generator=g))
        self.m.v_cache[:, :, :L].copy_(torch.randn(self.m.v_cache[:, :, :L].shape, generator=g))
        self.m._seq = L
        self.row = torch.cat([torch.tensor([ref.model.AUDIO_GEN_SLOT_TOKEN_ID]),
                              torch.randint(0, 1024, (32,), generator=g)]).view(1, 1, 33)
        self.kind = "reference"
        self.sample_desc = (f"reference moss_tts_lite.model.MossTTSModel on the host cores (torch CPU, bf16, "
                            f"{self.cores} threads): one audio-phase decode step = step(row) + text_logits_2way + "
                            f"audio_logits over all {c['n_layers']} layers at cache length {L + 1}+ "
                            f"({self.DISTINCT} distinct layer weight sets cycled over the layers)")

    def sample(self) -> float:
        import torch
        with torch.inference_mode():
            t0 = time.perf_counter()
            h = self.m.step(self.row)
            self.m.text_logits_2way(h)
            self.m.audio_logits(h)
            return time.perf_counter() - t0


class CpuOracleStep:
    """Fallback when the reference package is absent: the numpy oracle (the
    CPU restatement of the reference decoder) over all 36 layers at the
    configuration-2 shapes (fp32 BLAS on effective weights; four distinct
    layer weight sets cycled over the layers), embedding and audio-phase
    heads, cache length 129."""

    DISTINCT = 4

    def __init__(self, threads: int, steps: int):
        import numpy as np
        from oracle import step as ost
        from oracle.bf16 import f32_to_bf16
        try:
            from threadpoolctl import threadpool_limits
            self._limits = threadpool_limits(threads)
        except Exception:  # noqa: BLE001
            self._limits = None
        self.cores = threads
        c = CFG
        H, D = c["hidden"], c["head_dim"]
        rng = np.random.default_rng(1)

        def r(*shape):
            return f32_to_bf16((rng.standard_normal(shape, dtype=np.float32) * np.float32(c["std"])))
        one = lambda n: f32_to_bf16(np.ones(n, np.float32))  # noqa: E731
        w = {"language_model.embed_tokens.weight": np.zeros((c["vocab"], H), np.uint16),
             "language_model.norm.weight": one(H)}
        for li in range(self.DISTINCT):
            p = f"language_model.layers.{li}"
            w[f"{p}.input_layernorm.weight"] = one(H)
            w[f"{p}.post_attention_layernorm.weight"] = one(H)
            w[f"{p}.self_attn.q_proj.weight"] = r(c["n_heads"] * D, H)
            w[f"{p}.self_attn.k_proj.weight"] = r(c["n_kv"] * D, H)
            w[f"{p}.self_attn.v_proj.weight"] = r(c["n_kv"] * D, H)
            w[f"{p}.self_attn.o_proj.weight"] = r(H, c["n_heads"] * D)
            w[f"{p}.self_attn.q_norm.weight"] = one(D)
            w[f"{p}.self_attn.k_norm.weight"] = one(D)
            w[f"{p}.mlp.gate_proj.weight"] = r(c["inter"], H)
            w[f"{p}.mlp.up_proj.weight"] = r(c["inter"], H)
            w[f"{p}.mlp.down_proj.weight"] = r(H, c["inter"])
        for i in range(32):
            w[f"emb_ext.{i}.weight"] = r(1025, H)
            w[f"lm_heads.{i + 1}.weight"] = r(1025, H)
        w["lm_heads.0.weight"] = np.zeros((c["vocab"], H), np.uint16)
        self.ost = ost
        self.om = ost.OracleModel(w, max_seq_len=c["prompt_len"] + steps + 8, fp32_linears=True)
        self.om.seq = c["prompt_len"]
        self.row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
        self.kind = "port"
        self.sample_desc = (f"numpy oracle decode step at the configuration-2 shapes on {threads} BLAS threads: all "
                            f"{c['n_layers']} layers ({self.DISTINCT} distinct weight sets cycled), fp32 products "
                            f"on effective weights, embedding + audio-phase heads, cache length {c['prompt_len'] + 1}")

    def sample(self) -> float:
        om, ost = self.om, self.ost
        t0 = time.perf_counter()
        h = om.embed_rows(self.row.reshape(1, -1))
        for li in range(CFG["n_layers"]):
            h = om.layer(li % self.DISTINCT, h, om.seq)
        hf = ost.rms_norm(h, om.final_norm)
        om.text_logits_2way(hf)
        om.audio_logits(hf)
        return time.perf_counter() - t0


def cpu_step_runner(steps: int):
    """The reference's own decoder on CPU when its package is present, else
    the oracle port; all host cores."""
    threads = _host_threads()
    try:
        return CpuRefStep(threads, steps)
    except Exception:  # noqa: BLE001
        return CpuOracleStep(threads, steps)


def cpu_baseline(reps: int = 8):
    """(steps/s, cores, kind, sample description) of the CPU decode step:
    median of `reps` timed steps after two warm-up steps."""
    cs = cpu_step_runner(reps + 2)
    cs.sample()
    cs.sample()
    per_step = statistics.median(cs.sample() for _ in range(reps))
    return 1.0 / per_step, cs.cores, cs.kind, cs.sample_desc + f", median of {reps} steps"


def cpu_linears(shapes, reps: int = 5):
    """CPU baseline of W4 linears as the reference computes them on the host:
    moss_tts_lite.gptq.effective_weight (dequantise the codes and (scale,
    zero) to fp32) followed by the matmul, per projection, all host cores;
    median of `reps` runs of the whole list.  Returns (seconds, threads, kind)."""
    import torch
    threads = _host_threads()
    torch.set_num_threads(threads)
    ref = _ref_package()
    g = torch.Generator().manual_seed(2)
    cases = []
    for K, N in shapes:
        q = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
        s = torch.rand(N, K // 128, generator=g) * 0.01 + 1e-3
        mn = -8 * s
        qsz = torch.stack([s, mn + 8.0 * s], -1).bfloat16().transpose(0, 1).contiguous()
        cases.append((q, qsz, torch.randn(1, K, generator=g)))
    if ref is not None:
        eff = ref.gptq.effective_weight
        kind = "reference"
    else:
        from oracle.w4 import ref_effective_weight

        def eff(q, qsz, g):
            return torch.from_numpy(ref_effective_weight(q.numpy(), qsz.view(torch.int16).numpy().view("uint16"), g))
        kind = "port"

    def run():
        t0 = time.perf_counter()
        for q, qsz, x in cases:
            x @ eff(q, qsz, 128).t()
        return time.perf_counter() - t0
    run()
    return statistics.median(run() for _ in range(reps)), threads, kind


# --------------------------------------------------- configurations 0 and 1
CFG1_SHAPES = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
               ("gate", 4096, 12288), ("up", 4096, 12288), ("down", 12288, 4096)]


def _gptq_bytes(K: int, N: int, g: int = 128) -> int:
    """Algorithmic bytes of one AutoGPTQ W4 linear at batch 1: qweight + qzeros +
    scales + x + y."""
    return K * N // 2 + (K // g) * N // 2 + (K // g) * N * 2 + 2 * K + 2 * N


def _gptq_linear(dev, K: int, N: int, gen, g: int = 128):
    """A QuantLinear with the benchmark's distributions (codes and zeros
    uniform 0..15: random 32-bit words; scales |N(0,1)| * 0.01 + 1e-3 fp16),
    generated on the device."""
    import torch
    from moss_tts_lite_b200.quant import QuantLinear
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // 8, N), generator=gen, device=dev, dtype=torch.int32)
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (K // g, N // 8), generator=gen, device=dev, dtype=torch.int32)
    sc = (torch.randn(K // g, N, generator=gen, device=dev).abs() * 0.01 + 1e-3).half()
    return QuantLinear.from_tensors(qw, qz, sc, group_size=g)


def _graph_time(body, reps: int = 5) -> float:
    """Seconds per replay of a CUDA graph of `body` (warmed up; CUDA events)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e-3 / reps


def time_cfg0_cfg1(dev, cpu: bool):
    """Configuration 0 (one AutoGPTQ W4 linear 4096 -> 12288 at batch 1) and
    configuration 1 (one layer's seven W4 GPTQ projections) through
    QuantLinear.  Device: launches chained in a CUDA graph over several weight
    copies (inputs larger than L2), achieved = algorithmic bytes / time.
    End to end: QuantLinear.forward on a pinned host activation, the output
    copied back, synchronised per call.  CPU: the reference's
    effective_weight + matmul on the host cores."""
    import torch
    peak, peak_kind = _peaks()
    gen = torch.Generator(device=dev).manual_seed(0)
    out = {}
    # ---- configuration 0
    K, N = 4096, 12288
    lins = [_gptq_linear(dev, K, N, gen) for _ in range(8)]            # 209 MB > L2
    x = torch.randn(1, K, generator=gen, device=dev).to(torch.bfloat16)
    y = torch.empty(1, N, dtype=torch.bfloat16, device=dev)

    def body0():
        for i in range(64):
            lins[i % 8].w.linear(x, out=y)
    t0 = _graph_time(body0) / 64
    b0 = _gptq_bytes(K, N)
    xh = torch.randn(1, K).to(torch.bfloat16).pin_memory()
    yh = torch.empty(1, N, dtype=torch.bfloat16).pin_memory()
    for _ in range(5):
        yh.copy_(lins[0](xh.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize()
    reps = 200
    ts = time.perf_counter()
    for i in range(reps):
        yh.copy_(lins[i % 8](xh.to(dev, non_blocking=True)), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e0 = (time.perf_counter() - ts) / reps
    out["cfg0"] = {"workload": "cfg0: AutoGPTQ W4A16 linear 4096 -> 12288, g128, batch 1 (QuantLinear)",
                   "us_per_launch": t0 * 1e6, "bytes_per_launch": b0, "achieved_gbs": b0 / t0 / 1e9,
                   "frac": b0 / t0 / 1e9 / peak, "peak_gbs": peak, "peak_kind": peak_kind,
                   "timing": "64 launches in one CUDA graph over 8 weight copies (209 MB > L2)",
                   "e2e_us_per_call": e2e0 * 1e6,
                   "e2e": "QuantLinear.forward: pinned host x -> device, linear, y -> pinned host, synchronised"}
    del lins
    # ---- configuration 1
    layers = [[_gptq_linear(dev, k, n, gen) for _, k, n in CFG1_SHAPES] for _ in range(4)]   # 402 MB > L2
    xs = {k: torch.randn(1, k, generator=gen, device=dev).to(torch.bfloat16) for k in (4096, 12288)}
    ys = {n: torch.empty(1, n, dtype=torch.bfloat16, device=dev) for n in (1024, 4096, 12288)}

    def body1():
        for i in range(16):
            for lin, (_, k, n) in zip(layers[i % 4], CFG1_SHAPES):
                lin.w.linear(xs[k], out=ys[n])
    t1 = _graph_time(body1) / 16
    b1 = sum(_gptq_bytes(k, n) for _, k, n in CFG1_SHAPES)
    out["cfg1"] = {"workload": "cfg1: one layer's seven AutoGPTQ W4A16 projections (q, k, v, o, gate, up, down), "
                               "g128, batch 1, seven QuantLinear launches",
                   "us_per_layer": t1 * 1e6, "bytes_per_layer": b1, "achieved_gbs": b1 / t1 / 1e9,
                   "frac": b1 / t1 / 1e9 / peak, "peak_kind": peak_kind,
                   "timing": "16 layers in one CUDA graph over 4 layer copies (402 MB > L2)"}
    del layers
    torch.cuda.empty_cache()
    if cpu:
        s0, th, kind = cpu_linears([(K, N)])
        s1, _, _ = cpu_linears([(k, n) for _, k, n in CFG1_SHAPES])
        out["cfg0"]["cpu_baseline"] = {"us_per_call": s0 * 1e6, "cores": th, "kind": kind,
                                       "sample": "moss_tts_lite.gptq.effective_weight + matmul, median of 5"}
        out["cfg1"]["cpu_baseline"] = {"us_per_layer": s1 * 1e6, "cores": th, "kind": kind,
                                       "sample": "effective_weight + matmul per projection, median of 5"}
    return out


def reference_gpu_rate(dev, steps: int, warmup: int):
    """The reference's own W4 fast path on this GPU (the 5x denominator):
    moss_tts_lite.model.MossTTSModel + fast.FastMossTTS(quant='w4', g128,
    tinygemm) + generate_fast(greedy) on the same synthetic model and prompt;
    steps/s from generate_fast's own per-step CUDA-event stats after
    `warmup` steps.  None when the reference package is absent."""
    import torch
    ref = _ref_package()
    if ref is None:
        return None
    import moss_tts_lite.fast as rfast
    w = synth_weights(dev, CFG["seed"])
    model = ref.model.MossTTSModel(w, device=dev, dtype=torch.bfloat16, max_seq_len=MAX_SEQ)
    del w
    fast = rfast.FastMossTTS(model, quant="w4", w4_group_size=CFG["group_size"])
    st = {}
    res = rfast.generate_fast(fast, {"input_ids": make_prompt(CFG["seed"]).to(dev)},
                              max_new_tokens=warmup + steps + 1, greedy=True, watchdog=False, stats=st)
    ms = st["step_ms"][warmup:warmup + steps]
    out = {"value": 1000.0 / (sum(ms) / len(ms)), "unit": "steps/s", "steps": len(ms), "warmup": warmup,
           "steps_generated": res.n_steps,
           "what": "reference moss_tts_lite FastMossTTS(quant='w4', g128, tinygemm) + generate_fast(greedy), "
                   "same synthetic model and prompt, this GPU, its per-step CUDA-event stats"}
    del fast, model
    torch.cuda.empty_cache()
    return out


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
    """--impl reference: the reference's own decoder on the host cores (its
    MossTTSModel on device='cpu' when the package is present under
    baseline/_ref, else the numpy oracle port), all host threads whatever
    OMP_NUM_THREADS says; rank 0 only (the other ranks return at once).
    One step = one audio-phase decode step over all 36 layers."""
    if ctx.rank != 0:
        return
    cs = cpu_step_runner(args.steps + max(1, args.warmup))
    for _ in range(max(1, args.warmup)):
        cs.sample()
    secs = [cs.sample() for _ in range(args.steps)]
    v = len(secs) / sum(secs)
    line = {"metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if cs.kind == "reference" else "f32", "data": "synthetic",
            "config": {"workload": "cfg2: full synthetic MOSS-TTS-shaped W4 decode step, batch 1",
                       "model": "synthetic MOSS-TTS (36L, h4096, 32/8 heads, ffn 12288)"},
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": cs.cores, "kind": cs.kind,
                             "sample": cs.sample_desc},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_gemv_shapes():
    """Device time per W4 GEMV launch of each projection of the decode step
    (q|k|v, o, gate|up, down): 36 launches of one projection over the 36
    layers' weights in one CUDA graph (weights streaming from HBM), and the
    fit t = fixed + bytes / rate over the four shapes."""
    import numpy as np
    import torch
    dev = torch.device("cuda", 0)
    fast = build_fast(dev, seed=CFG["seed"], max_seq=256)
    eng, m = fast.engine, fast.m
    res = {}
    for name, res_epi in (("qkv", 0), ("o", 1), ("gu", 0), ("down", 1)):
        def body():
            for li in range(m.n_layers):
                lyr, L = m.layers[li], eng.lins[li]
                if name == "qkv":
                    L["qkv"](eng.h, eng.qkv, norm_weight=lyr["input_layernorm"])
                elif name == "o":
                    L["o"](eng.attn, eng.h, residual=eng.h)
                elif name == "gu":
                    L["gu"](eng.h, eng.act, norm_weight=lyr["post_attention_layernorm"], swiglu=True)
                else:
                    L["down"](eng.act, eng.h, residual=eng.h)
        t = _graph_time(body, reps=10) / m.n_layers
        w = eng.lins[0][name].w
        nout = w.N // 2 if name == "gu" else w.N
        nbytes = w.tiles.numel() + 2 * w.K + 2 * nout + (2 * w.N if res_epi else 0)
        res[name] = {"us": t * 1e6, "bytes": nbytes, "gbs": nbytes / t / 1e9}
    x = np.array([v["bytes"] for v in res.values()], np.float64)
    y = np.array([v["us"] for v in res.values()], np.float64)
    b, a = np.polyfit(x, y, 1)
    print(json.dumps({"profile": "w4 gemv per projection (36 chained launches each)", "per_shape": res,
                      "fit_fixed_us": a, "fit_rate_tbs": 1e-6 / b if b > 0 else None}))


def profile_chain():
    """Device time of the persistent W4 chain (mtl_w4_chain) per launch: the
    four-phase o -> gate|up -> down -> q|k|v chain over the 36 layers'
    weights in one graph, and one-phase chains of each projection (weights
    streaming from HBM), beside the one-launch-per-linear GEMV."""
    import torch
    from moss_tts_lite_b200 import kernels
    from moss_tts_lite_b200.model import RMS_EPS
    dev = torch.device("cuda", 0)
    fast = build_fast(dev, seed=CFG["seed"], max_seq=256)
    eng, m = fast.engine, fast.m
    if eng.strips is None:
        raise SystemExit("the chain is not enabled for this model")
    bar, g, n = eng.chain_bar, eng.chain_g, m.n_layers
    out = {}

    def chains(names):
        def body():
            for li in range(n):
                kernels.w4_chain([eng._phase(li, nm) for nm in names], g, bar[li], RMS_EPS)
        return body
    out["o,gu,down,qkv"] = _graph_time(chains(("o", "gu", "down", "qkv")), reps=10) / n * 1e6
    for nm in ("qkv", "o", "gu", "down"):
        out[nm] = _graph_time(chains((nm,)), reps=10) / n * 1e6
    print(json.dumps({"profile": "w4 chain us per launch (36 launches over the layers' weights)", "us": out}))


def profile_chain_rows(streams: int = 16):
    """Device time per launch of the batched persistent chain (mtl_w4_chain_rows,
    `streams` rows) over the 36 layers' strip weights, four-phase and
    one-phase, beside the batched attention launch at cache 256."""
    import torch
    from moss_tts_lite_b200 import kernels
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    from moss_tts_lite_b200.model import RMS_EPS
    dev = torch.device("cuda", 0)
    fast = build_fast(dev, seed=CFG["seed"], max_seq=512)
    bt = BatchedFastMossTTS(fast, streams, max_seq=512, chain=True)
    m, g, n = fast.m, fast.engine.chain_g, fast.m.n_layers
    bt.pos.fill_(256)
    out = {}

    def chains(names):
        def body():
            for li in range(n):
                kernels.w4_chain_rows([bt._phase(li, nm) for nm in names], g, bt.chain_bar[li], RMS_EPS)
        return body
    out["o,gu,down,qkv"] = _graph_time(chains(("o", "gu", "down", "qkv")), reps=5) / n * 1e6
    for nm in ("qkv", "o", "gu", "down"):
        out[nm] = _graph_time(chains((nm,)), reps=5) / n * 1e6

    def attn():
        for li in range(n):
            bt._attn(li)
    out["attn (cache 256)"] = _graph_time(attn, reps=5) / n * 1e6
    print(json.dumps({"profile": f"batched chain us per launch, {streams} rows", "us": out}))


def profile_chain_small(layers: int = 2, launches: int = 6, rows: int = 1):
    """A small ncu case for the persistent W4 chain: `layers` layers of
    configuration-2-shaped strip weights (random codes, ~205 MB, > L2 with
    two layers), `launches` four-phase chain launches cycling over them;
    with rows > 1 the batched chain (mtl_w4_chain_rows) on that many rows."""
    import torch
    from moss_tts_lite_b200 import kernels
    from moss_tts_lite_b200.quant import StripWeight
    dev = torch.device("cuda", 0)
    H, I, NQ, g = CFG["hidden"], CFG["inter"], CFG["n_heads"] * 128 + 2 * CFG["n_kv"] * 128, 128
    gen = torch.Generator(device=dev).manual_seed(0)

    def strip(K, N):
        q = torch.randint(0, 16, (N, K), device=dev, dtype=torch.uint8, generator=gen)
        qsz = torch.empty(K // g, N, 2, device=dev, dtype=torch.bfloat16)
        qsz[..., 0] = 0.01
        qsz[..., 1] = -0.005
        return StripWeight.from_ref(q, qsz, g)
    L = [{"o": strip(H, H), "gu": strip(H, 2 * I), "down": strip(I, H), "qkv": strip(H, NQ)} for _ in range(layers)]
    bf = torch.bfloat16
    lead = (rows,) if rows > 1 else ()
    h = torch.randn(*lead, H, device=dev, generator=gen).to(bf)
    attn = torch.randn(*lead, H, device=dev, generator=gen).to(bf)
    act = torch.empty(*lead, I, device=dev, dtype=bf)
    qkv = torch.empty(*lead, NQ, device=dev, dtype=bf)
    nw = torch.ones(H, device=dev, dtype=bf)
    launch = kernels.w4_chain_rows if rows > 1 else kernels.w4_chain
    def phases(w):
        return [{"w": w["o"], "x": attn, "y": h, "residual": h},
                {"w": w["gu"], "x": h, "y": act, "norm_w": nw, "swiglu": True},
                {"w": w["down"], "x": act, "y": h, "residual": h},
                {"w": w["qkv"], "x": h, "y": qkv, "norm_w": nw}]
    bar = torch.zeros(launches, 32, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(launches):
        if i == launches // 2:
            e0.record()
        launch(phases(L[i % layers]), g, bar[i], 1e-6)
    e1.record()
    torch.cuda.synchronize()
    n = launches - launches // 2
    print(json.dumps({"profile": "w4 chain small case", "layers": layers, "launches": launches, "rows": rows,
                      "us_per_launch_eager": e0.elapsed_time(e1) * 1e3 / n}))


def profile_gemv_ref(launches: int = 6):
    """Small case for ncu: the reference-format W4 linear of the decode step
    (RTN codes + bf16 (scale, zero) of a seeded N(0, 0.02) weight, 4096 ->
    12288, g128, batch 1, the configuration-0 shape) on cuda:0, `launches`
    launches over 4 weight copies (107 MB, > L2)."""
    import torch
    from moss_tts_lite_b200 import _lib, kernels
    from moss_tts_lite_b200.quant import W4Weight
    dev = torch.device("cuda", 0)
    K, N, g = 4096, 12288, 128
    gen = torch.Generator(device=dev).manual_seed(0)
    ws = []
    for _ in range(4):
        w = (torch.randn(N, K, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        q, qsz = kernels.rtn_quantize(w, g)
        ws.append(W4Weight.from_ref(q, qsz, g))
        del w, q, qsz
    x = torch.randn(1, K, generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty(1, N, dtype=torch.bfloat16, device=dev)
    for i in range(launches):
        ws[i % 4].linear(x, out=out)
    torch.cuda.synchronize()
    st = _lib.device_status()
    print(json.dumps({"profile": "w4_gemv reference format 4096 -> 12288", "launches": launches,
                      "bytes_per_launch": ws[0].tiles.numel() + 2 * K + 2 * N, "device_status": st}))
    if st != 0:
        raise SystemExit(1)


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


def profile_prefill(rows: int):
    """A prompt of `rows` rows (seeded random ids, last row AUDIO_START)
    prefilled through FastMossTTS.prefill on the configuration-2 model: two
    untimed calls, then one inside the NVTX range `mtl_timed` (the ncu
    launch-list case), timed with CUDA events."""
    import torch
    from moss_tts_lite_b200.model import AUDIO_START_TOKEN_ID, N_VQ
    dev = torch.device("cuda", 0)
    fast = build_fast(dev, seed=CFG["seed"], max_seq=max(rows + 8, 256))
    g = torch.Generator().manual_seed(3)
    ids = torch.zeros(1, rows, N_VQ + 1, dtype=torch.long)
    ids[0, :, 0] = torch.randint(0, 151643, (rows,), generator=g)
    ids[0, :, 1:] = torch.randint(0, 1024, (rows, N_VQ), generator=g)
    ids[0, -1, 0] = AUDIO_START_TOKEN_ID
    ids = ids.to(dev)
    for _ in range(2):
        fast.prefill(ids)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("mtl_timed")
    e0.record()
    fast.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    from moss_tts_lite_b200 import _lib
    print(json.dumps({"profile": f"prefill {rows} rows", "ms": e0.elapsed_time(e1),
                      "device_status": _lib.device_status()}))


def profile_attn(timed: bool = True, launches: int = 4, lengths=(136, 1024, 4096, 8191), splits: int = 16):
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
    print(json.dumps({"profile": "attn_decode cfg2", "splits": splits, "us_per_launch_in_graph": res,
                      "launches": launches, "device_status": st}))
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
    ap.add_argument("--no-reference-gpu", action="store_true", help="skip the in-process reference GPU arm")
    ap.add_argument("--no-cfg01", action="store_true", help="skip the configuration-0/1 linear measurements")
    ap.add_argument("--no-cfg3", action="store_true", help="skip the long-context sampled configuration-3 run")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the 16-stream batched configuration-4 run")
    ap.add_argument("--cfg4-tc", action="store_true", help="configuration 4 on tcgen05 tiles, one launch per linear")
    ap.add_argument("--profile-gemv", action="store_true", help="small config-0 GEMV case for ncu")
    ap.add_argument("--profile-gemv-ref", action="store_true", help="reference-format 4096->12288 GEMV (ncu case)")
    ap.add_argument("--profile-gemv-shapes", action="store_true", help="per-projection GEMV times and fixed-cost fit")
    ap.add_argument("--profile-chain", action="store_true", help="persistent W4 chain times per launch")
    ap.add_argument("--profile-chain-small", type=int, nargs="?", const=1, default=0,
                    help="2-layer W4 chain case (ncu); the value: activation rows (batched chain above 1)")
    ap.add_argument("--profile-chain-rows", type=int, default=0, help="batched chain times for this many rows")
    ap.add_argument("--profile-attn", action="store_true", help="decode attention alone (config 2 heads)")
    ap.add_argument("--profile-attn-launches", action="store_true", help="4 plain attention launches (ncu case)")
    ap.add_argument("--attn-len", type=int, default=136, help="cache length of the plain attention launches")
    ap.add_argument("--attn-splits", type=int, default=16, help="KV splits per head of --profile-attn")
    ap.add_argument("--profile-heads", action="store_true", help="text-head bf16 GEMV alone (ncu case)")
    ap.add_argument("--profile-cfg4", action="store_true", help="2 batched configuration-4 steps in an NVTX range")
    ap.add_argument("--profile-prefill", type=int, default=0, help="prefill of this many prompt rows (ncu case)")
    args = ap.parse_args()
    if args.profile_heads:
        profile_heads()
        return
    if args.profile_cfg4:
        profile_cfg4()
        return
    if args.profile_prefill:
        profile_prefill(args.profile_prefill)
        return
    if args.profile_gemv:
        profile_gemv()
        return
    if args.profile_gemv_ref:
        profile_gemv_ref()
        return
    if args.profile_gemv_shapes:
        profile_gemv_shapes()
        return
    if args.profile_chain:
        profile_chain()
        return
    if args.profile_chain_small:
        profile_chain_small(rows=args.profile_chain_small)
        return
    if args.profile_chain_rows:
        profile_chain_rows(args.profile_chain_rows)
        return
    if args.profile_attn or args.profile_attn_launches:
        lengths = (args.attn_len,) + tuple(L for L in (136, 1024, 4096, 8191) if L != args.attn_len)
        profile_attn(timed=args.profile_attn, lengths=lengths, splits=args.attn_splits)
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
    steps, warmup = args.steps, max(3, args.warmup)
    # the reference's own W4 fast path on this GPU first (rank 0), freed before ours is built
    ref_gpu = None
    if ctx.rank == 0 and not args.no_reference_gpu:
        ref_gpu = reference_gpu_rate(dev, steps=min(steps, 40), warmup=5)
    ctx.barrier()
    t_build = time.time()
    fast = build_fast(dev, seed=CFG["seed"] + ctx.rank)
    prompt = make_prompt(CFG["seed"] + ctx.rank)
    fast.prefill(prompt.to(dev))
    fast.capture()
    build_s = time.time() - t_build
    ms, clocks = time_decode_loop(fast, steps, warmup, ctx)
    ms = ctx.max(ms)
    ms_per_step = ms / steps
    value = ctx.world * steps / (ms * 1e-3)
    bytes_per_launch, s_per_launch, launches = time_w4_gemvs(fast)
    e2e, e2e_steps, e2e_relaunches, e2e_mix = time_e2e(fast, prompt.to("cpu"), steps, warmup)
    e2e_all = ctx.max(-(e2e or 0.0))  # slowest rank
    e2e_val = ctx.world * (-e2e_all) if e2e else None
    peak, peak_kind = _peaks()
    achieved = bytes_per_launch / s_per_launch / 1e9
    chained = fast.engine.strips is not None
    traffic = _ncu_traffic("w4_chain_traffic.json" if chained else "w4_gemv_traffic.json")
    single = ctx.world == 1
    cfg01 = None
    if ctx.rank == 0 and not args.no_cfg01:
        cfg01 = time_cfg0_cfg1(dev, cpu=single and not args.no_cpu_baseline)
    cfg3 = None
    if not args.no_cfg3:
        cfg3 = time_cfg3(fast)
        cfg3_e2e = ctx.max(-(cfg3["e2e_steps_per_s"] or 0.0))
        cfg3["e2e_steps_per_s_all_gpus"] = ctx.world * (-cfg3_e2e)
    cfg4 = None
    if not args.no_cfg4:
        cfg4 = time_cfg4(fast, tc=args.cfg4_tc)
        cfg4_ms = ctx.max(cfg4["device_ms_per_step"])
        cfg4["frames_per_s_all_gpus"] = ctx.world * cfg4["streams"] * 1e3 / cfg4_ms
        cfg4["n_gpus"] = ctx.world
    cpu = None
    if ctx.rank == 0 and single and not args.no_cpu_baseline:
        v, cores, kind, sample = cpu_baseline()
        cpu = {"value": v, "unit": "steps/s", "cores": cores, "kind": kind, "sample": sample}
    if ctx.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": ctx.world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2: full synthetic MOSS-TTS-shaped W4 decode step, batch 1",
                       "model": "synthetic MOSS-TTS (36L, h4096, 32/8 heads x128, ffn 12288, vocab 151936 + "
                                "32x1025 codebooks, RTN W4 g128, random-init seed 0)",
                       "global_batch": ctx.world, "seq_len": CFG["prompt_len"],
                       "parallelism": f"replicas{ctx.world}",
                       "phase": "audio (2-way text head + 32 audio heads), greedy tokens fed back on device",
                       "l2": "inputs larger than L2 (~3.9 GB of weights per step)",
                       "weights": "int4 codes + bf16 (scale, zero) per 128-group; operand bf16((q-8)*scale+zero) "
                                  "as the reference's int4 GEMM; activations bf16, fp32 accumulate",
                       "build_s": round(build_s, 1)},
            # per step: the 33 decisions come back to the host (pinned, 264 B);
            # the next input row is built on the device from them (as the
            # reference builds current_input_ids on the device), so no
            # per-step h2d copy; the prompt crosses once per call
            "e2e": {"value": e2e_val, "unit": "steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 33 * 8, "h2d_prompt_bytes": int(prompt.numel()) * 8,
                    "api": "moss_tts_lite_b200.fast.generate_fast(greedy=True)",
                    "steps_generated": e2e_steps, "speculation_relaunches": e2e_relaunches,
                    "phase_mix": e2e_mix,
                    "note": "next input row built on the device from the read-back decisions (no per-step h2d)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         # ncu DRAM bytes of the committed capture, scaled by its
                         # traffic/algorithmic ratio to the average step launch
                         "traffic": (bytes_per_launch * traffic["traffic_over_algorithmic"]
                                     if traffic else None),
                         "kernel": ("w4_chain_kernel (37 launches per step: q|k|v of layer 0, then o -> gate|up "
                                    "-> down -> next q|k|v per layer)" if chained else
                                    "w4_gemv_kernel (144 launches per step: q|k|v, o, gate|up, down x 36)"),
                         "bytes_per_launch": bytes_per_launch, "us_per_launch": s_per_launch * 1e6},
            "gpu_launches": steps * ((2 + 2 * CFG["n_layers"]) if chained else (1 + 5 * CFG["n_layers"])
                                     + 2 + 1),
            "clocks": clocks,
        }
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
            line["reference_gpu"]["ratio_device"] = (value / ctx.world) / ref_gpu["value"]
            if e2e_val:
                line["reference_gpu"]["ratio_e2e"] = (e2e_val / ctx.world) / ref_gpu["value"]
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if cfg01 is not None:
            line.update(cfg01)
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
