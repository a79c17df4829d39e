"""B200-native (sm_100a) rebuild of moss-tts-lite's W4 decode hot path.

Host-side mirror of the reference interface (moss_tts_lite.gptq / fast /
model / sampling) over the C ABI of ``libmtl_b200.so``.  Import a submodule
(``moss_tts_lite_b200.quant``, ``.fast`` ...) to load the library; there is
no CPU or PyTorch fallback for any op.
"""
__version__ = "0.1.0"
