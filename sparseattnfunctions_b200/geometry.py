"""Token geometry of CogVideoX-style DiT attention.

The reference hard-codes the CogVideoX-2B layout (226 text tokens, then a
13 x 30 x 45 (t, h, w) video grid: MergeAttention.py:16,26-31,
merge_unmerge.py:83,121, SmartAttention.py:15-26, mask_related.py:100-101)
and the 1.5-5B one (224 text, 11 x 48 x 85: combined_attn.py:17-41,
partern_attention.py:10-16).  Every shape constant here is derived from one
``VideoGeometry`` instead.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class VideoGeometry:
    text_len: int = 226
    frames: int = 13
    height: int = 30
    width: int = 45

    @property
    def frame_len(self) -> int:
        return self.height * self.width

    @property
    def video_len(self) -> int:
        return self.frames * self.frame_len

    @property
    def seq_len(self) -> int:
        return self.text_len + self.video_len

    def text_blocks(self, block: int) -> int:
        """Blocks that contain at least one text token (text comes first)."""
        return math.ceil(self.text_len / block)

    def num_blocks(self, block: int) -> int:
        return math.ceil(self.seq_len / block)


COGVIDEOX_2B = VideoGeometry(226, 13, 30, 45)
COGVIDEOX_2B_LONG = VideoGeometry(226, 25, 30, 45)   # 33976 tokens
COGVIDEOX_15_5B = VideoGeometry(224, 11, 48, 85)
