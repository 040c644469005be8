"""Prompt -> token ids (reference behaviour: python/minisgl/tokenizer/tokenize.py:10-31).
A list of chat messages goes through the tokenizer's chat template with a generation prompt."""

from __future__ import annotations

from typing import List

import torch


class TokenizeManager:
    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer

    def encode_one(self, text) -> torch.Tensor:
        if isinstance(text, list):
            ids = self.tokenizer.apply_chat_template(text, tokenize=True, add_generation_prompt=True)
            if isinstance(ids, dict) or hasattr(ids, "input_ids"):
                ids = ids["input_ids"]
        else:
            ids = self.tokenizer.encode(text)
        return torch.tensor(list(ids), dtype=torch.int32)

    def tokenize(self, msgs) -> List[torch.Tensor]:
        return [self.encode_one(m.text) for m in msgs]
