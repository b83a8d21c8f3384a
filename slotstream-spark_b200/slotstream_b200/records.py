"""Expert record byte layout, derived from (hidden, inter, gs).

One routed expert is one contiguous record of nine pieces in this order:
gate.w, gate.s, gate.b, up.w, up.s, up.b, down.w, down.s, down.b
(slotstream_spark/kernels/moe_gemv_affine.py:11-13, :21-25; tools/repack_experts.py:1-8).

* ``*.w``: MLX affine 4-bit codes, int32 words, row-major [n, k/8]; element i of a row sits in
  bits [4*(i%8), 4*(i%8)+4) of word i//8, little endian (kernels/affine_ref.py:3-19).
* ``*.s`` / ``*.b``: bf16 scale and bias, row-major [n, k/gs]; w = q*s + b.
* gate/up are [inter, hidden] (n = inter, k = hidden); down is [hidden, inter].

The reference hard-codes the model's 2560/640 shape (RECORD_BYTES = 2,764,800); this module computes
the same offsets for any shape, so 2048/512 gives a 1,769,472-byte record with the identical piece order.
"""
from dataclasses import dataclass

EXPERTS_PER_LAYER = 512          # map[layer * 512 + e] (kernels/moe_gemv_affine.py:68)
MAP_LAYERS = 49                  # map tables hold 49 * 512 entries (kernels/moe_gemv_affine.py:117)


@dataclass(frozen=True)
class RecordLayout:
    hidden: int
    inter: int
    gs: int = 64

    def __post_init__(self):
        if self.hidden % self.gs or self.inter % self.gs:
            raise ValueError(f"hidden={self.hidden} and inter={self.inter} must be multiples of gs={self.gs}")
        if self.gs not in (32, 64):
            raise ValueError(f"gs must be 32 or 64, got {self.gs}")

    # piece sizes in bytes
    @property
    def w_bytes(self) -> int:          # one 4-bit matrix of inter x hidden (gate, up and down have the same count)
        return self.inter * self.hidden // 2

    @property
    def sb_bytes(self) -> int:         # one bf16 scale (or bias) matrix
        return self.inter * self.hidden // self.gs * 2

    @property
    def proj_bytes(self) -> int:
        return self.w_bytes + 2 * self.sb_bytes

    @property
    def record_bytes(self) -> int:
        return 3 * self.proj_bytes

    def offsets(self):
        """(O_GATE_W, O_GATE_S, O_GATE_B, O_UP_W, O_UP_S, O_UP_B, O_DOWN_W, O_DOWN_S, O_DOWN_B)."""
        out = []
        for p in range(3):
            base = p * self.proj_bytes
            out += [base, base + self.w_bytes, base + self.w_bytes + self.sb_bytes]
        return tuple(out)

    def piece_shapes(self):
        """[(n, k)] of gate, up, down."""
        return [(self.inter, self.hidden), (self.inter, self.hidden), (self.hidden, self.inter)]


BASELINE_LAYOUT = RecordLayout(2048, 512, 64)     # BASELINE config-[0]: hidden 2048, intermediate 512, gs 64
REFERENCE_LAYOUT = RecordLayout(2560, 640, 64)    # the reference model's shape (kernels/moe_gemv_affine.py:21-22)
