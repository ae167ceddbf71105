"""oracle/medusa.py -- CPU restatement of the reference's Medusa heads.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of
spec_medusa_topk; the shipped library never uses it.

Restates crates/speculate/src/methods/medusa.rs:
* MedusaHeadModule::forward (:564-584): per residual block
  x <- x + SiLU(linear(x)) (weight [H][H] and bias [H]), then the output
  projection linear_no_bias(hidden -> vocab);
* MedusaHeadsCandle::forward / top_k_per_head (:706-734): every head reads
  the same hidden row; top_k_indices (:477-487) per head.

Math in float64 over BF16 weights.  Each linear's input is rounded to BF16,
where the device's GEMV operand is (the reference computes the heads in the
checkpoint's BF16), so the comparison tolerance only covers accumulation
order and the f32 residual stream.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

from .accept import top_k_indices
from .eagle import bf16_round, bits_to_f32


class MedusaOracle:
    def __init__(self, res_w: Sequence[Sequence[np.ndarray]], res_b: Sequence[Sequence[np.ndarray]],
                 out_w: Sequence[np.ndarray]):
        self.res_w = [[bits_to_f32(w).astype(np.float64) for w in head] for head in res_w]
        self.res_b = [[np.asarray(b, dtype=np.float64) for b in head] for head in res_b]
        self.out_w = [bits_to_f32(w).astype(np.float64) for w in out_w]

    @staticmethod
    def _op(x: np.ndarray) -> np.ndarray:
        return bf16_round(np.asarray(x, dtype=np.float32)).astype(np.float64)

    def forward(self, hidden: np.ndarray) -> List[np.ndarray]:
        """medusa.rs:706-708 / :564-584: one logits row per head."""
        rows = []
        for ws, bs, wo in zip(self.res_w, self.res_b, self.out_w):
            x = np.asarray(hidden, dtype=np.float64)
            for w, b in zip(ws, bs):
                y = w @ self._op(x) + b
                x = x + y / (1.0 + np.exp(-y))
            rows.append(wo @ self._op(x))
        return rows

    def top_k_per_head(self, hidden: np.ndarray, k: int) -> Tuple[List[List[int]], List[np.ndarray]]:
        """medusa.rs:713-734: the top-k ids of every head and its logits row."""
        rows = self.forward(hidden)
        return [top_k_indices(r, k) for r in rows], rows
