"""Streaming detokenization (reference behaviour: python/minisgl/tokenizer/detokenize.py:35-111).

Per request we keep the generated ids and two offsets: ``prefix`` (ids before this point are
already rendered in ``text``) and ``emitted`` (characters of ``text`` already sent). Each step
decodes the ids from a small look-back window so merges across token boundaries render correctly,
holds back output ending in an incomplete UTF-8 sequence (U+FFFD), and otherwise only releases
whole words (or CJK characters / newlines) until the request finishes. EOS is not rendered.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List

_REPLACEMENT = "�"


def _is_cjk(ch: str) -> bool:
    cp = ord(ch)
    return (
        0x4E00 <= cp <= 0x9FFF or 0x3400 <= cp <= 0x4DBF or 0x20000 <= cp <= 0x2A6DF
        or 0x2A700 <= cp <= 0x2B73F or 0x2B740 <= cp <= 0x2B81F or 0x2B820 <= cp <= 0x2CEAF
        or 0xF900 <= cp <= 0xFAFF or 0x2F800 <= cp <= 0x2FA1F
    )


def printable_prefix(text: str) -> str:
    """Longest prefix of ``text`` that cannot change when more tokens arrive."""
    if not text or text.endswith("\n"):
        return text
    if _is_cjk(text[-1]):
        return text
    if len(text) > 1 and _is_cjk(text[-2]):
        return text[:-1]
    return text[: text.rfind(" ") + 1]


@dataclass
class _Stream:
    ids: List[int] = field(default_factory=list)
    text: str = ""      # stable rendered text
    prefix: int = 0     # ids[:prefix] are part of `text`
    window: int = 0     # ids[window:prefix] are re-decoded as left context
    emitted: int = 0    # characters of the output already sent


class DetokenizeManager:
    def __init__(self, tokenizer) -> None:
        self.tokenizer = tokenizer
        self.eos_token_id = tokenizer.eos_token_id
        self.streams: Dict[int, _Stream] = {}

    def detokenize(self, msgs) -> List[str]:
        ctx_ids, full_ids = [], []
        for m in msgs:
            st = self.streams.setdefault(m.uid, _Stream())
            if not m.eos:
                st.ids.append(m.next_token)
            ctx_ids.append(st.ids[st.window : st.prefix])
            full_ids.append(st.ids[st.window :])
        ctx_txt = self.tokenizer.batch_decode(ctx_ids)
        full_txt = self.tokenizer.batch_decode(full_ids)
        out: List[str] = []
        for m, ctx, full in zip(msgs, ctx_txt, full_txt):
            st = self.streams[m.uid]
            new = full[len(ctx):]
            if new and not new.endswith(_REPLACEMENT):
                st.text += new
                st.window, st.prefix = st.prefix, len(st.ids)
                visible = st.text
            else:  # incomplete: release only what cannot change (everything, once finished)
                visible = st.text + (new.rstrip(_REPLACEMENT) if m.finished else printable_prefix(new))
            if m.finished:
                del self.streams[m.uid]
            out.append(visible[st.emitted:])
            st.emitted = max(st.emitted, len(visible))
        return out
