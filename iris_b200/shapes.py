"""Model shapes of the benchmark configurations and the host-side shape
arithmetic the reference's importer performs before inference starts.

Integer restatements (Python integers are exact) of:
- det_num::mistral::attention_scale_q32 (crates/det-num/src/mistral.rs:148-160),
- det_num::mistral::yarn_inverse_frequencies (mistral.rs:185-214),
- det_num::convert::f32_to_act / f32_to_acc (crates/det-num/src/convert.rs:4-97),
- the Gemma scalars of crates/model/import/src/gemma.rs:740-755.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from typing import List, Optional


def attention_scale_q32(head_dim: int) -> int:
    """floor(2^32 / sqrt(head_dim)) by binary search on the square."""
    target = (1 << 64) // max(head_dim, 1)
    lo, hi = 0, (1 << 32) - 1
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if mid * mid <= target:
            lo = mid
        else:
            hi = mid - 1
    return lo


def _isqrt(v: int) -> int:
    return math.isqrt(v)  # floor square root, as integer_sqrt (mistral.rs:162-176)


def yarn_inverse_frequencies(base: int, pairs: int, factor: int, low: int, high: int) -> Optional[List[int]]:
    if pairs <= 0 or pairs & (pairs - 1) or base == 0 or factor == 0 or high <= low:
        return None
    root = base << 32
    for _ in range(pairs.bit_length() - 1):
        root = _isqrt(root << 32)
    step = ((1 << 64) + root // 2) // root
    span = high - low
    plain = 1 << 32
    out = []
    for pair in range(pairs):
        kept = min(max(high - pair, 0), span)
        num = plain * (span + (factor - 1) * kept)
        den = factor * span
        out.append((num + den // 2) // den)
        plain = (plain * step + (1 << 31)) >> 32
    return out


def _f32_fixed(x: float, frac: int, max_pos: int, max_neg: int) -> int:
    bits = struct.unpack("<I", struct.pack("<f", x))[0]
    neg = bits >> 31
    eb, fb = (bits >> 23) & 0xFF, bits & 0x7FFFFF
    if eb == 0 and fb == 0:
        return 0
    sig, ex = (fb, -149) if eb == 0 else ((1 << 23) | fb, eb - 150)
    se = ex + frac
    maxm = max_neg if neg else max_pos
    if se >= 0:
        mag = maxm if sig > (maxm >> se) else sig << se
    else:
        q, r, half = sig >> -se, sig & ((1 << -se) - 1), 1 << (-se - 1)
        mag = min(q + 1 if r > half or (r == half and q & 1) else q, maxm)
    if neg:
        return -max_neg if mag >= max_neg else -mag
    return mag


def f32_to_act(x: float) -> int:
    return max(min(_f32_fixed(x, 16, 2**31 - 1, 2**31), 2**31 - 1), -(2**31))


def f32_to_acc(x: float) -> int:
    return max(min(_f32_fixed(x, 32, 2**63 - 1, 2**63), 2**63 - 1), -(2**63))


@dataclass
class MistralConfig:
    """mistral-dense shape (crates/inference/artifacts/src/direct.rs:267-287)."""
    name: str
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_base: int = 1_000_000
    max_positions: int = 32768
    eps: float = 1e-5
    tied: bool = False
    family: str = "mistral"
    # YaRN (factor, low, high) from an imported config.json; None: plain RoPE
    yarn: Optional[tuple] = None

    @property
    def norm_eps(self) -> int:
        return f32_to_acc(self.eps)

    @property
    def freqs(self) -> List[int]:
        # plain RoPE: YaRN factor 1 reduces to base^(-j / pairs)
        factor, low, high = self.yarn or (1, 0, 1)
        return yarn_inverse_frequencies(self.rope_base, self.head_dim // 2, factor, low, high)

    @property
    def scale_q32(self) -> int:
        return attention_scale_q32(self.head_dim)


@dataclass
class GemmaConfig:
    """gemma-dense shape (direct.rs:241-262) plus its per-layer derivations."""
    name: str
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    ple_width: int
    sliding_window: int = 0
    layer_types: List[str] = field(default_factory=list)   # "sliding_attention" | "full_attention"
    num_kv_shared_layers: int = 0
    rope_base_sliding: int = 10_000
    rope_base_full: int = 1_000_000
    partial_rotary: float = 0.25
    softcap: float = 0.0
    eps: float = 1e-6
    layer_scalars: Optional[List[int]] = None
    tied: bool = True
    family: str = "gemma"

    def types(self) -> List[str]:
        return self.layer_types or ["sliding_attention"] * self.layers

    @property
    def norm_eps(self) -> int:
        return f32_to_acc(self.eps)

    def is_sliding(self, l: int) -> bool:
        return self.types()[l] == "sliding_attention"

    def window(self, l: int) -> int:
        return self.sliding_window if self.is_sliding(l) else 0

    def rope(self, l: int):
        """(base Acc bits, rotary_dim, freq_base_dim) (direct/src/model.rs:819-828)."""
        if self.is_sliding(l):
            return self.rope_base_sliding << 32, self.head_dim, self.head_dim
        q16 = round(self.partial_rotary * 65536)
        return self.rope_base_full << 32, (self.head_dim * q16) // 65536, self.head_dim

    def kv_donor(self, l: int) -> int:
        """direct/src/model.rs:830-844."""
        first_shared = max(self.layers - self.num_kv_shared_layers, 0)
        if self.num_kv_shared_layers == 0 or l < first_shared:
            return -1
        t = self.types()[l]
        for cand in range(first_shared - 1, -1, -1):
            if self.types()[cand] == t:
                return cand
        return -1

    def donor_candidates(self):
        donors = sorted({self.kv_donor(l) for l in range(self.layers) if self.kv_donor(l) >= 0})
        return (donors[0] if donors else -2, donors[1] if len(donors) > 1 else -3)

    @property
    def embedding_scale(self) -> int:  # import/src/gemma.rs:746-749
        return f32_to_act(math.sqrt(float(self.hidden)))

    @property
    def ple_embedding_scale(self) -> int:
        return f32_to_act(math.sqrt(float(self.ple_width)))

    @property
    def ple_projection_scalar(self) -> int:
        return f32_to_act(float(struct.unpack("<f", struct.pack("<f", float(self.hidden) ** -0.5))[0]))

    @property
    def ple_input_scale(self) -> int:
        return f32_to_act(2.0 ** -0.5)

    @property
    def softcap_bits(self) -> int:
        return f32_to_act(self.softcap) if self.softcap else 0


# ---- the benchmark configurations (BASELINE.json "configs") ---------------

def tiny_gemma() -> GemmaConfig:
    """Config 1: L2, H256, 4q/1kv, d64, GeGLU 1024, V8192, tied, RoPE 10000.
    Every layer sliding with a window (96) that covers the 32+64 positions, so
    attention is full; PLE width 64; no softcap."""
    return GemmaConfig("tiny-gemma", layers=2, hidden=256, ffn=1024, heads=4, kv_heads=1, head_dim=64,
                       vocab=8192, ple_width=64, sliding_window=96, rope_base_sliding=10_000)


def gemma_2b() -> GemmaConfig:
    """Config 3: L18, H2048, 8q/1kv, d256, GeGLU 16384, V256000, PLE 256, all
    sliding (window 768), base 10000, softcap 30."""
    return GemmaConfig("gemma-2b-arch", layers=18, hidden=2048, ffn=16384, heads=8, kv_heads=1, head_dim=256,
                       vocab=256000, ple_width=256, sliding_window=768, rope_base_sliding=10_000, softcap=30.0)


def mistral_7b() -> MistralConfig:
    """Config 4: L32, H4096, 32q/8kv, d128, SwiGLU 14336, V32000 (untied),
    RoPE base 1e6; the 4096 sliding window is a no-op at these lengths."""
    return MistralConfig("mistral-7b-arch", layers=32, hidden=4096, ffn=14336, heads=32, kv_heads=8,
                         head_dim=128, vocab=32000, rope_base=1_000_000, max_positions=32768)


def parity_mistral() -> MistralConfig:
    """The shape of the reference's parity bundle (model-bundles/parity-mistral:
    4 layers, H128, F2048, 4q/2kv, d32, V512, tied) with plain RoPE."""
    return MistralConfig("parity-mistral", layers=4, hidden=128, ffn=2048, heads=4, kv_heads=2, head_dim=32,
                         vocab=512, rope_base=1_000_000, max_positions=16384, tied=True)


def tp_mistral() -> MistralConfig:
    """A small mistral-dense shape for the tensor-parallel tests: its kv heads
    (8), FFN blocks (1024 / 32) and vocabulary (1024) divide 2, 4 and 8 ranks;
    the 7B model's group of 4 query heads a kv head."""
    return MistralConfig("tp-mistral", layers=2, hidden=256, ffn=1024, heads=32, kv_heads=8, head_dim=32,
                         vocab=1024, rope_base=1_000_000, max_positions=16384, tied=True)


def parity_gemma() -> GemmaConfig:
    """A small gemma-dense shape with what the reference's parity bundle
    exercises: a sliding window of 16, two K/V-sharing layers, a full layer
    with partial rotary, PLE 32 and softcap 1.0 (model-bundles/parity-gemma)."""
    return GemmaConfig("parity-gemma", layers=4, hidden=128, ffn=512, heads=4, kv_heads=1, head_dim=32,
                       vocab=512, ple_width=32, sliding_window=16,
                       layer_types=["sliding_attention", "full_attention", "sliding_attention", "full_attention"],
                       num_kv_shared_layers=2, rope_base_sliding=10_000, rope_base_full=1_000_000,
                       partial_rotary=0.25, softcap=1.0, layer_scalars=[0, 3 << 15, 0, 1 << 16])


CONFIGS = {c.name: c for c in (tiny_gemma(), gemma_2b(), mistral_7b(), parity_mistral(), parity_gemma(),
                               tp_mistral())}
