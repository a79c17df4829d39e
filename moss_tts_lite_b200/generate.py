"""Generation result container (moss_tts_lite/generate.py:21-26)."""
from dataclasses import dataclass

import torch


@dataclass
class GenResult:
    text_ids: torch.Tensor
    audio_frames: torch.Tensor
    finished: bool
    n_steps: int
