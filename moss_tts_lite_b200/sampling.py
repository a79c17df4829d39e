"""Token sampling for generate_fast on the sm_100a kernels.

Greedy decisions (``do_sample=False``, sampling.py:84-85 of the reference)
are first-index argmaxes computed by ``mtl_argmax_rows`` /
``mtl_argmax_masked``.  Temperature / top-k / top-p sampling
(sampling.py:70-98) runs in the fused per-row sampling kernel.
"""
from __future__ import annotations


class sample_rows:  # noqa: N801 - namespace of the two sampled decisions
    """Sampled text / audio decisions of one generate_fast step."""

    @staticmethod
    def text(fast, is_audio, time_step, temperature, top_k, top_p, gen):
        raise NotImplementedError("sampled text decisions need the fused sampling kernel (not built yet)")

    @staticmethod
    def audio(fast, smask, temperature, top_k, top_p, penalty, prev_audio, gen):
        raise NotImplementedError("sampled audio decisions need the fused sampling kernel (not built yet)")
