"""Host control flow of generate_fast on the CPU: the state machine and the
pipelined driver (moss_tts_lite_b200.fsm) against the reference's own
generate_fast loop (moss_tts_lite/fast.py:342-610), both driving the same
deterministic fake model whose logits depend on the fed input row and the
cache position.  Greedy decisions, so both loops must produce the same
tokens, step count and watchdog record.  The fake's logits are biased so that
the trajectories pass through the text phase, audio start, the delay / end
pattern, silence watchdog stops and im_end stops; the speculative driver must
relaunch on each of those mode changes and still match."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from moss_tts_lite_b200 import fsm
from moss_tts_lite_b200.model import (AUDIO_PAD_CODE, AUDIO_START_TOKEN_ID, AUDIO_VOCAB, IM_END_TOKEN_ID,
                                      N_VQ, TEXT_VOCAB)

H = 4  # fake hidden: [two-way 0, two-way 1, pos, row hash]


def _row_hash(row) -> int:
    h = 1469598103
    for v in row:
        h = (h * 1000003 + int(v) + 7) % 2147483629
    return h


def _hidden(pos: int, row, bias: dict) -> torch.Tensor:
    rh = _row_hash(row)
    delay = (rh + pos) % bias["delay_every"] == 0
    two = (0.0, 5.0) if delay else (5.0, 0.0)
    return torch.tensor([[two[0], two[1], float(pos), float(rh)]], dtype=torch.float32)


class _FakeModel:
    """The heads the reference loop calls, as functions of the fake hidden."""

    def __init__(self, bias, max_seq_len=4096):
        self.device = torch.device("cpu")
        self.max_seq_len = max_seq_len
        self.head_2way = torch.zeros(2, H)
        self.head_2way[0, 0] = 1.0
        self.head_2way[1, 1] = 1.0
        self.bias = bias

    def _gen(self, h):
        h = h.reshape(-1)
        g = torch.Generator().manual_seed(int(h[3]) * 7919 + int(h[2]))
        return g, int(h[2]), int(h[3])

    def text_logits(self, h):
        g, pos, rh = self._gen(h)
        lt = torch.randn(TEXT_VOCAB, generator=g)
        if (rh + 3 * pos) % self.bias["start_every"] == 0:
            lt[AUDIO_START_TOKEN_ID] = 50.0
        if pos > self.bias["im_end_after"] and (rh + pos) % self.bias["im_end_every"] == 0:
            lt[IM_END_TOKEN_ID] = 60.0
        return lt

    def audio_logits(self, h):
        g, pos, rh = self._gen(h)
        la = torch.randn(N_VQ, AUDIO_VOCAB, generator=g)
        if (rh + pos) % self.bias["silence_every"] < self.bias["silence_len"]:
            la[0, 9] = 50.0        # a low-energy channel-0 code (watchdog silence)
        la[:, AUDIO_PAD_CODE] = float("-inf")
        return la


class _Hidden:
    def __init__(self, h):
        self.last_hidden = h


class _FakeFast:
    """FastMossTTS surface of the reference loop over the fake model."""

    def __init__(self, bias):
        self.m = _FakeModel(bias)
        self.bias = bias
        self.ids_row = torch.zeros(1, 1, N_VQ + 1, dtype=torch.long)
        self.lt_buf = torch.full((TEXT_VOCAB,), float("-inf"))

    def prefill(self, input_ids):
        L = input_ids.shape[1]
        h = _hidden(L, input_ids[0, -1].tolist(), self.bias)
        return _Hidden(h.view(1, 1, H).expand(1, L, H).contiguous())

    def capture(self):
        pass

    def heads(self, h):
        return self.m.text_logits(h), self.m.audio_logits(h), F.linear(h[0], self.m.head_2way)

    def step(self, row, pos, audio2=False):
        h = _hidden(pos, self.ids_row.view(-1).tolist(), self.bias)
        lt, la, two = self.heads(h)
        return lt, la, h, two


def _argmax_excl(x: torch.Tensor, excluded) -> int:
    x = x.clone()
    for e in excluded:
        x[e] = float("-inf")
    return int(torch.argmax(x))


class _FakeOps:
    """This package's device side (feed kernel, head graph, decision kernels)
    restated over the fake model, with the same two-slot decision ring."""

    def __init__(self, fast: _FakeFast, prompt):
        self.fast = fast
        self.prompt = prompt
        self.dec = [[0] * (N_VQ + 1), [0] * (N_VQ + 1)]
        self.launches = 0

    def _feed(self, dec, p: fsm.StepPlan):
        from moss_tts_lite_b200.model import AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID
        text = p.text_const
        if p.text_mode == fsm.TEXT_TWO_WAY:
            text = AUDIO_GEN_SLOT_TOKEN_ID if dec[0] == 0 else AUDIO_DELAY_SLOT_TOKEN_ID
        elif p.text_mode == fsm.TEXT_ID:
            text = dec[0]
        row, k = [text], 0
        for j in range(N_VQ):
            if p.smask >> j & 1:
                row.append(dec[1 + (k if p.sample_audio else j)])
                k += 1
            else:
                row.append(AUDIO_PAD_CODE)
        return row

    def launch(self, t, plan, prev, pos):
        self.launches += 1
        f = self.fast
        if t == 0:
            h = f.prefill(self.prompt).last_hidden[:, -1]
        else:
            row = self._feed(self.dec[(t - 1) & 1], prev)
            f.ids_row.view(-1).copy_(torch.tensor(row))
            h = _hidden(pos, row, f.bias)
        lt, la, two = f.heads(h)
        out = list(self.dec[t & 1])
        if plan.greedy_audio:
            out[1:] = [int(v) for v in torch.argmax(la, -1)]
        if plan.greedy_text:
            out[0] = _argmax_excl(two if plan.text_two else lt, plan.excluded)
        assert not (plan.sample_text or plan.sample_audio)
        self.dec[t & 1] = out

    def fetch(self, t):
        return list(self.dec[t & 1])


BIASES = {
    "audio_long": dict(delay_every=37, start_every=5, im_end_after=10 ** 9, im_end_every=3, silence_every=50,
                       silence_len=2),
    "text_then_audio": dict(delay_every=23, start_every=11, im_end_after=60, im_end_every=17, silence_every=40,
                            silence_len=3),
    "silence_stop": dict(delay_every=10 ** 6, start_every=3, im_end_after=10 ** 9, im_end_every=3,
                         silence_every=12, silence_len=9),
    "im_end_early": dict(delay_every=7, start_every=4, im_end_after=35, im_end_every=2, silence_every=30,
                         silence_len=1),
}


def _prompt(L, seed, audio_start):
    rng = np.random.default_rng(seed)
    ids = torch.zeros(1, L, N_VQ + 1, dtype=torch.long)
    ids[0, :, 0] = torch.from_numpy(rng.integers(0, 151000, L))
    ids[0, :, 1:] = torch.from_numpy(rng.integers(0, 1024, (L, N_VQ)))
    if audio_start:
        ids[0, -1, 0] = AUDIO_START_TOKEN_ID
    return ids


def _mine(bias, prompt, max_new, pipelined, **wd):
    fast = _FakeFast(bias)
    cfg = fsm.GenConfig.make(False, False, wd.get("watchdog", True), wd.get("watchdog_silence_frames"),
                             wd.get("watchdog_max_segment_frames"), None)
    st = fsm.FsmState.from_prompt(prompt[0, :, 0].tolist())
    ops = _FakeOps(fast, prompt)
    r = fsm.drive(ops, st, cfg, max_new, int(prompt.shape[1]), pipelined=pipelined)
    return r, ops


@pytest.mark.parametrize("case", sorted(BIASES))
@pytest.mark.parametrize("audio_start", [True, False])
@pytest.mark.parametrize("wd", [dict(watchdog=True, watchdog_silence_frames=4),
                                dict(watchdog=True, watchdog_silence_frames=2, watchdog_max_segment_frames=8),
                                dict(watchdog=False)])
def test_fsm_matches_reference_loop(case, audio_start, wd):
    ref = pytest.importorskip("moss_tts_lite.fast")
    bias = BIASES[case]
    prompt = _prompt(9, seed=len(case), audio_start=audio_start)
    max_new = 160
    theirs = ref.generate_fast(_FakeFast(bias), {"input_ids": prompt}, max_new_tokens=max_new, greedy=True, **wd)
    for pipelined in (False, True):
        r, ops = _mine(bias, prompt, max_new, pipelined, **wd)
        assert r.n_steps == theirs.n_steps, (pipelined, r.n_steps, theirs.n_steps)
        assert r.text_steps == theirs.text_ids.tolist()
        assert r.audio_steps == theirs.audio_frames.tolist()
        assert bool(r.state.wd_stats) == theirs.watchdog_triggered
        assert r.state.wd_reason == theirs.watchdog_reason
        assert r.state.wd_stats == theirs.watchdog_stats
        finished = bool(r.state.is_stopping) or bool(r.state.wd_stats)
        assert finished == theirs.finished
        if not pipelined:
            assert ops.launches == r.n_steps and r.relaunches == 0
        else:
            # one launch per step, plus one per mode change and the speculated tail
            assert ops.launches == r.n_steps + r.relaunches + int(r.speculative_tail)


def test_fsm_trajectories_cover_mode_changes():
    """The fake biases do reach the transitions the speculation must undo."""
    from moss_tts_lite_b200.model import AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID
    seen = set()
    for case, bias in BIASES.items():
        for audio_start in (True, False):
            r, _ = _mine(bias, _prompt(9, seed=len(case), audio_start=audio_start), 160, True,
                         watchdog=True, watchdog_silence_frames=4)
            seen.update(t for t in r.text_steps if t in (AUDIO_START_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID,
                                                          AUDIO_END_TOKEN_ID, IM_END_TOKEN_ID))
            if r.state.wd_reason:
                seen.add(r.state.wd_reason)
            assert r.relaunches >= 0
    assert {AUDIO_START_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID, IM_END_TOKEN_ID,
            "silence"} <= seen, seen


def test_plan_is_decision_free_and_advance_is_pure():
    st = fsm.FsmState(is_audio=True, al=40)
    cfg = fsm.GenConfig.make(False, False, True)
    p = fsm.make_plan(st, 5, cfg)
    assert p == fsm.make_plan(st, 5, cfg) and p.smask == (1 << N_VQ) - 1 and p.text_mode == fsm.TEXT_TWO_WAY
    s2, text, audio, stop = fsm.advance(st, p, 1, list(range(N_VQ)), 4, cfg)
    assert st.dl == fsm.INT64_MAX and s2.dl == 1 and not stop     # delay slot starts the delay pattern
    assert audio == list(range(N_VQ))
    p2 = fsm.make_plan(s2, 6, cfg)
    assert p2.text_mode == fsm.TEXT_FORCED and p2.smask == ((1 << N_VQ) - 1) & ~1
