"""Host control flow of generate_fast: the delay-pattern state machine of the
reference loop (moss_tts_lite/fast.py:342-610) split into a pure
``make_plan`` / ``advance`` pair, and the pipelined driver that keeps the next
decode step in flight while the host decides the current one.

``make_plan(state, t)`` fixes everything the device does in step t before its
decisions are known: which head graph runs (text or audio two-way), the forced
text token of the delay / end pattern, which audio channels are decided
(smask, fast.py:520), which decisions are greedy or sampled, the exclusions
and the Philox offset.  ``advance(state, plan, decisions)`` is the rest of the
loop body: the text decision, the audio row, the watchdog
(fast.py:547-564) and the al / dl counters (fast.py:566-578).

The driver (``drive``) launches step t+1 speculatively, with the plan that
follows from step t when its text decision keeps the current mode (GEN slot
in audio, an ordinary token in text), before it reads step t's decisions back.
The next input row itself never needs a guess: the device builds it from step
t's decisions (``mtl_feed_row``) with the feed arguments of plan t, which are
exact.  When the real plan of step t+1 differs from the speculated one (a
mode change: audio start, delay slot, end, stop, watchdog), step t+1 is
launched again with the real plan; everything the speculative launch wrote is
rewritten (the input row, pos, the K/V row at pos, the logits and the
decision slot), so the result is the same as a loop without speculation.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

from .model import (AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_PAD_CODE,
                    AUDIO_START_TOKEN_ID, IM_END_TOKEN_ID, N_VQ, PAD_TOKEN_ID)

INT64_MAX = 9223372036854775807
WD_LOW_ENERGY_CH0 = frozenset(
    (9, 60, 109, 123, 163, 209, 216, 365, 399, 402, 421, 580, 715, 734,
     774, 795, 827, 888, 890, 936, 971, 996, 1001))
WD_SEGMENT_FLOOR = 640
WD_SEGMENT_BACKSTOP_RUN = 32
# the greedy text exclusions of the text phase (fast.py:427-429, 505-511)
PRE_EXCLUDE0 = (PAD_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID)

TEXT_FORCED, TEXT_TWO_WAY, TEXT_ID = 0, 1, 2


@dataclass(frozen=True)
class GenConfig:
    """Loop constants of one generate_fast call (fast.py:403-444)."""

    text_do_sample: bool
    audio_do_sample: bool
    watchdog: bool = True
    wd_floor: int = WD_SEGMENT_FLOOR
    wd_sil: int = 64
    max_requested_pause_s: float | None = None

    @staticmethod
    def make(text_do_sample: bool, audio_do_sample: bool, watchdog: bool, watchdog_silence_frames=None,
             watchdog_max_segment_frames=None, max_requested_pause_s=None) -> "GenConfig":
        wd_floor = watchdog_max_segment_frames if watchdog_max_segment_frames is not None else WD_SEGMENT_FLOOR
        wd_sil = watchdog_silence_frames if watchdog_silence_frames is not None else 64
        if max_requested_pause_s is not None and max_requested_pause_s > 0:
            wd_sil = max(wd_sil, math.ceil((max_requested_pause_s + 2.0) * 12.5))
        return GenConfig(text_do_sample, audio_do_sample, watchdog, wd_floor, wd_sil, max_requested_pause_s)


@dataclass
class FsmState:
    """The loop variables of fast.py:418-444 that carry from step to step."""

    is_audio: bool
    al: int = 0
    dl: int = INT64_MAX
    is_stopping: bool = False
    wd_stop: bool = False
    wd_reason: str = ""
    wd_silent_run: int = 0
    wd_peak_segment: int = 0
    wd_stats: dict = field(default_factory=dict)
    step_offset: int = 0     # Philox offset counter of the sampled decisions

    @staticmethod
    def from_prompt(col0: list) -> "FsmState":
        """fast.py:411-418: continuation detection from the prompt's text column."""
        seq_len = len(col0)
        is_cont = col0[-1] in (AUDIO_START_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID)
        hits = [i for i, c in enumerate(col0) if c == AUDIO_START_TOKEN_ID]
        start_idx = hits[-1] if hits else -1
        al = seq_len - start_idx if (is_cont and start_idx != -1) else 0
        return FsmState(is_audio=is_cont and start_idx != -1, al=al)


@dataclass(frozen=True)
class StepPlan:
    """What the device does in one step before its decisions are known."""

    time_step: int
    audio2: bool            # head graph: two-way text head (audio phase) or the text head
    is_audio: bool          # audio phase for the text decision (after a forced END)
    audio_off: bool         # the forced END ends the audio phase
    text_mode: int          # TEXT_FORCED (text_const) / TEXT_TWO_WAY (0 -> GEN, else DELAY) / TEXT_ID
    text_const: int
    smask: int              # bit j: audio channel j is decided this step
    greedy_text: bool
    text_two: bool          # greedy text source: the two-way logits (else the text logits)
    excluded: tuple         # greedy text exclusions
    greedy_audio: bool
    sample_text: bool
    sample_audio: bool
    offset: int             # Philox step offset of the sampled decisions

    @property
    def smask_list(self) -> list:
        return [bool(self.smask >> j & 1) for j in range(N_VQ)]


def make_plan(st: FsmState, t: int, cfg: GenConfig) -> StepPlan:
    """The decisions-independent part of one loop iteration (fast.py:460-545)."""
    text_const, audio_off = PAD_TOKEN_ID, False
    if st.wd_stop:
        if st.dl == INT64_MAX or st.dl < N_VQ:
            text_const = AUDIO_DELAY_SLOT_TOKEN_ID
        else:
            text_const, audio_off = AUDIO_END_TOKEN_ID, True
    elif not st.is_stopping and st.dl < N_VQ:
        text_const = AUDIO_DELAY_SLOT_TOKEN_ID
    elif not st.is_stopping and st.dl == N_VQ:
        text_const, audio_off = AUDIO_END_TOKEN_ID, True
    is_audio = st.is_audio and not audio_off
    sampling_text = (not st.is_stopping) and (not st.wd_stop) and st.dl > N_VQ
    smask = 0
    for j in range(N_VQ):
        if st.al > j and (st.dl == INT64_MAX or j > st.dl - 1):
            smask |= 1 << j
    need_audio = smask != 0
    greedy_text = sampling_text and not cfg.text_do_sample
    greedy_audio = need_audio and not cfg.audio_do_sample
    text_two, excluded = True, ()
    if greedy_text or greedy_audio:
        if sampling_text and is_audio:
            excluded = (1,) if t == 0 else ()
        elif sampling_text:
            ex = list(PRE_EXCLUDE0)
            if t == 0:
                ex.append(AUDIO_DELAY_SLOT_TOKEN_ID)
            if t <= N_VQ:
                ex.append(IM_END_TOKEN_ID)
            text_two, excluded = False, tuple(sorted(set(ex)))
    sample_text = sampling_text and cfg.text_do_sample
    sample_audio = need_audio and cfg.audio_do_sample
    offset = st.step_offset + 1 if (sample_text or sample_audio) else st.step_offset
    text_mode = TEXT_FORCED
    if sampling_text:
        text_mode = TEXT_TWO_WAY if is_audio else TEXT_ID
    return StepPlan(t, st.is_audio, is_audio, audio_off, text_mode, text_const, smask, greedy_text, text_two,
                    excluded, greedy_audio, sample_text, sample_audio, offset)


def decode_raw(plan: StepPlan, raw: list) -> tuple[int, list]:
    """Decision slot [33] -> (text decision, per-channel audio decisions).
    Sampled audio decisions are compact over the decided channels."""
    if not plan.sample_audio:
        return raw[0], raw[1:1 + N_VQ]
    audio = [AUDIO_PAD_CODE] * N_VQ
    k = 0
    for j in range(N_VQ):
        if plan.smask >> j & 1:
            audio[j] = raw[1 + k]
            k += 1
    return raw[0], audio


def advance(st: FsmState, plan: StepPlan, text_dec: int, audio: list, n_steps: int,
            cfg: GenConfig) -> tuple[FsmState, int, list, bool]:
    """The decisions-dependent part of one loop iteration (fast.py:487-590):
    returns the next state, the row (next_text, next_audio) and whether the
    loop stops after this step."""
    s = replace(st)
    s.step_offset = plan.offset
    if plan.audio_off:
        s.is_audio = False
    next_text = plan.text_const
    if plan.text_mode == TEXT_TWO_WAY:
        next_text = AUDIO_GEN_SLOT_TOKEN_ID if int(text_dec) == 0 else AUDIO_DELAY_SLOT_TOKEN_ID
    elif plan.text_mode == TEXT_ID:
        next_text = int(text_dec)
    if next_text == AUDIO_START_TOKEN_ID:
        s.is_audio = True
    if next_text == IM_END_TOKEN_ID:
        s.is_stopping = True
    next_audio = [AUDIO_PAD_CODE] * N_VQ
    for j in range(N_VQ):
        if plan.smask >> j & 1:
            next_audio[j] = int(audio[j])
    if cfg.watchdog and not s.wd_stop and s.is_audio and s.dl == INT64_MAX:
        if next_audio[0] in WD_LOW_ENERGY_CH0:
            s.wd_silent_run += 1
        else:
            s.wd_silent_run = 0
        seg_bound = max(cfg.wd_floor, 2 * s.wd_peak_segment)
        if s.wd_silent_run >= cfg.wd_sil:
            s.wd_stop, s.wd_reason = True, "silence"
        elif s.al > seg_bound and s.wd_silent_run >= WD_SEGMENT_BACKSTOP_RUN:
            s.wd_stop, s.wd_reason = True, "max_segment"
        if s.wd_stop:
            s.wd_stats = {"reason": s.wd_reason, "step": n_steps + 1, "segment_frames": s.al,
                          "silent_run": s.wd_silent_run, "peak_completed_segment": s.wd_peak_segment,
                          "silence_threshold_frames": cfg.wd_sil, "segment_bound_frames": seg_bound,
                          "max_requested_pause_s": cfg.max_requested_pause_s}
    if next_text in (AUDIO_START_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID):
        s.al += 1
    if next_text == AUDIO_END_TOKEN_ID:
        s.wd_peak_segment = max(s.wd_peak_segment, s.al)
        s.wd_silent_run = 0
        s.al = 0
    if s.dl == INT64_MAX and next_text == AUDIO_DELAY_SLOT_TOKEN_ID:
        s.dl = 0
    if s.dl != INT64_MAX:
        s.dl += 1
    if s.dl > N_VQ:
        s.dl = INT64_MAX
    stop = s.is_stopping or (s.wd_stop and next_text == AUDIO_END_TOKEN_ID)
    return s, next_text, next_audio, stop


@dataclass
class DriveResult:
    state: FsmState
    text_steps: list
    audio_steps: list
    n_steps: int
    relaunches: int
    speculative_tail: bool   # a speculated step past the last one was launched


def drive(ops, st: FsmState, cfg: GenConfig, max_new_tokens: int, seq_len: int, pipelined: bool = True,
          on_step=None) -> DriveResult:
    """Run the loop over ``ops`` (``launch(t, plan, prev_plan, pos)`` enqueues
    step t: for t >= 1 the feed of its input row from step t-1's decisions
    with prev_plan's feed arguments, the head graph at ``pos``, and its
    decisions into slot t % 2; ``fetch(t)`` waits for step t and returns its
    decision slot as 33 ints).  Step t >= 1 runs at cache position
    seq_len + t - 1 (fast.py:466-468)."""
    text_steps: list = []
    audio_steps: list = []
    if max_new_tokens <= 0:
        return DriveResult(st, text_steps, audio_steps, 0, 0, False)
    plan = make_plan(st, 0, cfg)
    ops.launch(0, plan, None, seq_len)
    t, n_steps, relaunches = 0, 0, 0
    last_audio = [AUDIO_PAD_CODE] * N_VQ
    spec_tail = False
    while True:
        spec = None
        if pipelined and t + 1 < max_new_tokens:
            guess_text = 0 if plan.text_mode == TEXT_TWO_WAY else -1
            pst, _, _, pstop = advance(st, plan, guess_text, last_audio, n_steps, cfg)
            if not pstop:
                spec = make_plan(pst, t + 1, cfg)
                ops.launch(t + 1, spec, plan, seq_len + t)
        text_dec, audio = decode_raw(plan, ops.fetch(t))
        st, next_text, next_audio, stop = advance(st, plan, text_dec, audio, n_steps, cfg)
        text_steps.append(next_text)
        audio_steps.append(next_audio)
        n_steps += 1
        last_audio = next_audio
        if on_step is not None:
            on_step(t, plan)
        if stop or t + 1 >= max_new_tokens:
            spec_tail = spec is not None
            break
        nxt = make_plan(st, t + 1, cfg)
        if nxt != spec:
            relaunches += spec is not None
            ops.launch(t + 1, nxt, plan, seq_len + t)
        plan = nxt
        t += 1
    return DriveResult(st, text_steps, audio_steps, n_steps, relaunches, spec_tail)
