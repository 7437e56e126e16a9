"""mockbird_b200 -- B200 (sm_100a) KV-ring / RoPE / attention path of Mockbird's
MOSS-TTS-Nano decoder, behind the C ABI of include/mockbird_kv.h.

    from mockbird_b200 import KvRing
    ring = KvRing(capacity=512, streams=64, wrap=True)
    ctx = ring.append_attend(layer, streams, positions, qkv)   # one fused launch
"""
from .engine import Decoder, KvRing, LocalHead, MockbirdError, argmax_penalty  # noqa: F401
from ._lib import LIB_PATH, load  # noqa: F401

__all__ = ["Decoder", "KvRing", "LocalHead", "MockbirdError", "argmax_penalty", "LIB_PATH", "load"]
