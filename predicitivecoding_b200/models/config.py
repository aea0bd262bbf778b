"""Decoder configuration with the reference's field names and presets.

Reference: PredictiveCoding.LLM/Autograd/DecoderLM.cs:31-130 (``DecoderLmConfig``).
Field names follow the reference's PascalCase in the JSON form
(:meth:`DecoderLmConfig.to_json` / :meth:`from_json`) so configs written by one
side load in the other.  Two fields are extensions the reference never trained:
``ffn`` ("gelu" = the reference's dense GELU FFN with biases, "swiglu" = gated
SiLU FFN without biases, used by the GPT-2-small / 1.3B configs) and ``tie_io``
(kept False: the reference unties the embedding and the output head).
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Optional

_PASCAL = {
    "vocab": "Vocab", "dim": "Dim", "num_blocks": "NumBlocks", "num_heads": "NumHeads", "ff_dim": "FfDim",
    "max_seq": "MaxSeq", "dropout": "Dropout", "eps": "Eps", "num_loops": "NumLoops",
    "loop_exit_tau": "LoopExitTau", "mtp_weight": "MtpWeight", "mtp_horizon": "MtpHorizon",
    "block_pattern": "BlockPattern", "num_experts": "NumExperts", "moe_top_k": "MoeTopK",
    "moe_balance_weight": "MoeBalanceWeight", "use_plan": "UsePlan", "use_rms_norm": "UseRmsNorm",
    "use_rope": "UseRope", "ffn": "Ffn",
}


@dataclass(frozen=True)
class DecoderLmConfig:
    vocab: int
    dim: int
    num_blocks: int
    num_heads: int
    ff_dim: int
    max_seq: int
    dropout: float = 0.0
    eps: float = 1e-5
    num_loops: int = 1
    loop_exit_tau: float = 0.0
    mtp_weight: float = 0.0
    mtp_horizon: int = 2
    block_pattern: Optional[str] = None
    num_experts: int = 0
    moe_top_k: int = 1
    moe_balance_weight: float = 0.01
    use_plan: bool = False
    use_rms_norm: bool = False
    use_rope: bool = False
    ffn: str = "gelu"

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads

    def validate(self) -> None:
        """Same rules as DecoderLmConfig.Validate (DecoderLM.cs:54-90)."""
        if min(self.vocab, self.dim, self.num_blocks, self.num_heads, self.ff_dim, self.max_seq) <= 0:
            raise ValueError("All DecoderLmConfig sizes must be positive.")
        if self.dim % self.num_heads:
            raise ValueError(f"Dim ({self.dim}) must be divisible by NumHeads ({self.num_heads}).")
        if self.num_loops < 1:
            raise ValueError(f"NumLoops ({self.num_loops}) must be >= 1.")
        if self.loop_exit_tau < 0:
            raise ValueError("LoopExitTau must be >= 0 (0 disables the early exit).")
        if self.mtp_weight < 0:
            raise ValueError("MtpWeight must be >= 0 (0 disables multi-token prediction).")
        if self.mtp_weight > 0 and self.mtp_horizon < 2:
            raise ValueError("MtpHorizon must be >= 2 when MtpWeight is on (2 = predict t+2).")
        if self.block_pattern is not None:
            if len(self.block_pattern) != self.num_blocks:
                raise ValueError("BlockPattern length must equal NumBlocks.")
            for c in self.block_pattern:
                if c not in "AT":
                    raise ValueError(f"BlockPattern may only contain 'A' or 'T', found '{c}'.")
        if self.num_experts < 0:
            raise ValueError("NumExperts must be >= 0 (0 = dense feed-forward).")
        if self.num_experts > 0 and not (1 <= self.moe_top_k <= self.num_experts):
            raise ValueError(f"MoeTopK ({self.moe_top_k}) must be in [1, NumExperts ({self.num_experts})].")
        if self.moe_balance_weight < 0:
            raise ValueError("MoeBalanceWeight must be >= 0.")
        if self.use_rope and self.head_dim % 2:
            raise ValueError(f"UseRope needs an even head dim, got {self.head_dim}.")
        if (self.use_rms_norm or self.use_rope) and self.block_pattern is not None:
            raise ValueError("UseRmsNorm/UseRope are attention-only (BlockPattern must be null).")
        if self.ffn not in ("gelu", "swiglu"):
            raise ValueError(f"ffn must be 'gelu' or 'swiglu', got {self.ffn!r}.")

    # ---------------------------------------------------------------- presets
    @staticmethod
    def small(vocab: int, max_seq: int = 512) -> "DecoderLmConfig":
        """~30M-class preset (DecoderLM.cs:107): dim 384, 8 blocks, 6 heads, ffn 1536, RMSNorm+RoPE."""
        return DecoderLmConfig(vocab, 384, 8, 6, 1536, max_seq, use_rms_norm=True, use_rope=True)

    @staticmethod
    def base(vocab: int, max_seq: int = 1024) -> "DecoderLmConfig":
        """GPT-2-small-class preset (DecoderLM.cs:112): dim 768, 12 blocks, 12 heads, ffn 3072."""
        return DecoderLmConfig(vocab, 768, 12, 12, 3072, max_seq, use_rms_norm=True, use_rope=True)

    @staticmethod
    def byte_lm_4l() -> "DecoderLmConfig":
        """Byte LM: 4 layers, d 256, 4 heads, ctx 256, vocab 256, RMSNorm, RoPE, GELU 4x."""
        return DecoderLmConfig(256, 256, 4, 4, 1024, 256, use_rms_norm=True, use_rope=True, ffn="gelu")

    @staticmethod
    def gpt2_small_swiglu() -> "DecoderLmConfig":
        """124M-class decoder: 12 layers, d 768, 12 heads, ctx 1024, vocab 32000, SwiGLU 2048."""
        return DecoderLmConfig(32000, 768, 12, 12, 2048, 1024, use_rms_norm=True, use_rope=True, ffn="swiglu")

    @staticmethod
    def decoder_1p3b() -> "DecoderLmConfig":
        """1.3B decoder: 24 layers, d 2048, 16 heads, ctx 2048, vocab 32000, SwiGLU 5504."""
        return DecoderLmConfig(32000, 2048, 24, 16, 5504, 2048, use_rms_norm=True, use_rope=True, ffn="swiglu")

    def dense_parameter_formula(self) -> int:
        """Exact parameter count of a dense config (DecoderLM.cs:121-130; SwiGLU adds a third matrix)."""
        if self.num_experts > 0 or self.num_loops > 1 or self.mtp_weight > 0 or self.use_plan or self.block_pattern:
            raise ValueError("dense_parameter_formula only covers the plain dense-attention config.")
        norm_per_block = 2 * self.dim if self.use_rms_norm else 4 * self.dim
        if self.ffn == "gelu":
            ffn = 2 * self.dim * self.ff_dim + self.ff_dim + self.dim
        else:
            ffn = 3 * self.dim * self.ff_dim
        per_block = 4 * self.dim * self.dim + ffn + norm_per_block
        final_norm = self.dim if self.use_rms_norm else 2 * self.dim
        return 2 * self.vocab * self.dim + self.num_blocks * per_block + final_norm

    # ---------------------------------------------------------------- JSON
    def to_json(self) -> str:
        d = {}
        for k, v in dataclasses.asdict(self).items():
            if k == "ffn" and v == "gelu":
                continue  # the reference has no such field; omit the default
            d[_PASCAL[k]] = v
        return json.dumps(d)

    @staticmethod
    def from_json(s: str) -> "DecoderLmConfig":
        raw = json.loads(s)
        inv = {v: k for k, v in _PASCAL.items()}
        kw = {}
        for k, v in raw.items():
            name = inv.get(k, k)
            if name in DecoderLmConfig.__dataclass_fields__:
                kw[name] = v
        return DecoderLmConfig(**kw)

    def with_(self, **kw) -> "DecoderLmConfig":
        return dataclasses.replace(self, **kw)
