"""Hugging Face helpers: tokenizer, cached config and weight download
(reference: python/minisgl/utils/hf.py:17-52). Works offline on local directories."""

from __future__ import annotations

import functools
import json
import os
from typing import Any


def load_tokenizer(model_path: str):
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(model_path)
    if not getattr(tok, "chat_template", None):
        # some checkpoints keep the template in a side file
        side = os.path.join(model_path, "chat_template.json") if os.path.isdir(model_path) else None
        if side is None:
            try:
                from huggingface_hub import hf_hub_download

                side = hf_hub_download(repo_id=model_path, filename="chat_template.json")
            except Exception:
                side = None
        if side and os.path.exists(side):
            with open(side, encoding="utf-8") as f:
                tok.chat_template = json.load(f)["chat_template"]
    return tok


@functools.cache
def _load_config(model_path: str) -> Any:
    from transformers import AutoConfig

    return AutoConfig.from_pretrained(model_path)


def cached_load_hf_config(model_path: str):
    cfg = _load_config(model_path)
    return type(cfg)(**cfg.to_dict())  # fresh copy so callers may mutate


def download_hf_weight(model_path: str) -> str:
    if os.path.isdir(model_path):
        return model_path
    try:
        from huggingface_hub import snapshot_download

        return snapshot_download(model_path, allow_patterns=["*.safetensors"])
    except Exception as e:  # no network on most boxes
        raise ValueError(f"'{model_path}' is not a local directory and cannot be downloaded: {e}")
