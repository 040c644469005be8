"""minisgl: an LLM serving engine written for NVIDIA B200 (sm_100a).

Public entry points mirror the reference project's surface:
``python -m minisgl`` (OpenAI-compatible server / shell), ``minisgl.llm.LLM`` (offline API).
"""

__version__ = "0.1.0"
