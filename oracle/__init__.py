"""CPU oracle for the moss-tts-lite W4 decode hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
directory. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` (plus its ``--impl reference`` arm) may import it, and
they use it as the checker, never as the thing that is measured or shipped.

Modules:

* ``bf16``     - bfloat16 <-> float32 helpers with round-to-nearest-even.
* ``w4``       - int4 (AutoGPTQ and reference ``(q, qsz)``) unpack/dequant,
                 RTN quantisation, and the fp32 GEMV that the W4 linear must
                 match (moss_tts_lite/gptq.py, moss_tts_lite/fast.py).
* ``step``     - one decoder step of the reference model restated op by op
                 with the reference's bf16 rounding points
                 (moss_tts_lite/model.py, moss_tts_lite/fast.py).
* ``sampling`` - argmax / top-k / top-p / repetition penalty restated from
                 moss_tts_lite/sampling.py, plus the delay-pattern FSM of
                 moss_tts_lite/fast.py:generate_fast.

Pinning: every module is checked in ``tests/test_oracle_*.py`` against
golden vectors under ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by importing and running the reference package itself.
"""
