"""Row layout of the mixed decode + packed-prefill MoE call.

The reference runs one backbone over decode rows first and the packed prompt
rows second; the prompt segment has a fixed capacity whose tail is padding
(src/drama3/mixed_graph.py:33-50, packed_prefill.py:11-48). Each row carries a
slot: decode rows their request's slot, prompt rows their sequence's slot, the
padding a reserved slot (row_metadata, packed_prefill.py:58-77). Rows whose slot
is at or above the reserved boundary route with row 0's logits
(moe_input.py:32-36).

Prompt rows that repeat an earlier prompt's rows from position 0 produce the
same MoE output, so the MoE can run on a compact row set (row_reuse.py:45-105,
mixed_model.py:193-246): `keep` lists the rows the MoE runs on (padded to a
64-row bucket with row 0) and `inverse` names the compact row each full row
takes. `d3moe.ops.moe_layer(..., keep=, inverse=, row_slots=, padding_start=)`
consumes both in one call.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

# (decode rows, prefill capacity, prompt span, compact rows) of the prebuilt
# mixed graphs (src/drama3/row_reuse.py:9-15).
MIXED_ROW_REUSE_BUCKETS = (
    (64, 768, 256, 576),
    (64, 1024, 256, 832),
    (64, 1280, 256, 1088),
    (64, 1536, 256, 1088),
    (64, 1536, 256, 1344),
)


@dataclass(frozen=True)
class RowReusePlan:
    """packed_indices = keep [compact_rows] followed by inverse [decode_rows +
    prefill_capacity], like the reference's plan (row_reuse.py:18-42)."""

    decode_rows: int
    prefill_capacity: int
    compact_rows: int
    unique_rows: int
    prompt_lengths: tuple
    packed_indices: torch.Tensor
    prompt_bytes: tuple

    @property
    def keep(self) -> torch.Tensor:
        return self.packed_indices[: self.compact_rows]

    @property
    def inverse(self) -> torch.Tensor:
        return self.packed_indices[self.compact_rows:]

    @property
    def removed_rows(self) -> int:
        return self.decode_rows + self.prefill_capacity - self.compact_rows

    def matches_prompts(self, prompts) -> bool:
        """True only for the same prompts, byte for byte (a stale plan must not run)."""
        if tuple(len(p) for p in prompts) != self.prompt_lengths:
            return False
        for p, snap in zip(prompts, self.prompt_bytes):
            if p.device.type != "cpu" or p.dtype != torch.int64 or p.ndim != 2 or p.shape[1] != 11:
                return False
            if p.numpy().tobytes() != snap:
                return False
        return True


def _common_prefix(a: np.ndarray, b: np.ndarray) -> int:
    n = min(len(a), len(b))
    same = np.all(a[:n] == b[:n], axis=1)
    diff = np.flatnonzero(~same)
    return int(diff[0]) if len(diff) else n


def plan_row_reuse(prompts, decode_rows: int, prefill_capacity: int, compact_capacities):
    """Row ownership of the mixed call, or None when no compact bucket fits.

    Same contract as src/drama3/row_reuse.py:45-105: prompts are CPU int64
    [length, 11] rows packed after `decode_rows` decode rows. A prompt's first
    L rows alias the rows of the earlier prompt sharing the longest row prefix
    with it (the first such prompt on ties; rows are compared whole, up to the
    first difference), resolved to that prompt's own owners. Decode rows and
    the padding after the last prompt own themselves. The compact bucket is the
    smallest capacity >= the unique row count rounded up to 64; its spare rows
    repeat row 0."""
    if decode_rows < 1 or prefill_capacity < 1 or not 1 <= len(prompts) <= 8:
        raise ValueError("Invalid mixed row counts")
    for p in prompts:
        if p.device.type != "cpu" or p.dtype != torch.int64 or p.ndim != 2 or p.shape[1] != 11:
            raise ValueError("Row reuse requires CPU int64 prompts with eleven columns")
    lengths = tuple(len(p) for p in prompts)
    if min(lengths) < 3 or max(lengths) > 512 or sum(lengths) > prefill_capacity:
        raise ValueError("Prompts do not fit the mixed prefill capacity")
    full = decode_rows + prefill_capacity
    buckets = sorted(set(compact_capacities))
    for c in buckets:
        if c <= 0 or c % 64 or c > full - 256:
            raise ValueError("Compact buckets must be 64-aligned and remove at least 256 rows")
    if not buckets:
        return None
    arrays = [p.numpy() for p in prompts]
    owner = np.arange(full, dtype=np.int64)
    starts = []
    at = decode_rows
    for i, cur in enumerate(arrays):
        best, src = 0, -1
        for j in range(i):
            n = _common_prefix(cur, arrays[j])
            if n > best:
                best, src = n, j
        if best:
            owner[at:at + best] = owner[starts[src]:starts[src] + best]
        starts.append(at)
        at += len(cur)
    keep = np.flatnonzero(owner == np.arange(full))
    unique = len(keep)
    need = -(-unique // 64) * 64
    compact = next((c for c in buckets if c >= need), None)
    if compact is None:
        return None
    compact_of = np.zeros(full, dtype=np.int64)
    compact_of[keep] = np.arange(unique, dtype=np.int64)
    packed = np.zeros(compact + full, dtype=np.int64)
    packed[:unique] = keep
    packed[compact:] = compact_of[owner]
    return RowReusePlan(decode_rows, prefill_capacity, compact, unique, lengths,
                        torch.from_numpy(packed), tuple(a.tobytes() for a in arrays))


def packed_row_slots(decode_slots, lengths, sequence_slots, capacity: int) -> np.ndarray:
    """Slot of every row of the mixed call: the decode slots, then each prompt's
    rows with its sequence slot, then the trailing padding with the last
    sequence slot (the reserved padding slot), as row_metadata writes them
    (src/drama3/packed_prefill.py:58-77; boundaries from
    mixed_graph.py:41-50). `sequence_slots` has one slot per prompt plus the
    padding slot."""
    lengths = list(lengths)
    if len(sequence_slots) != len(lengths) + 1:
        raise ValueError("sequence_slots needs one slot per prompt and one for the padding")
    if sum(lengths) > capacity:
        raise ValueError("Prompts exceed packed prefill capacity")
    segs = lengths + [capacity - sum(lengths)]
    prompt_slots = np.repeat(np.asarray(sequence_slots, dtype=np.int64), segs)
    return np.concatenate([np.asarray(decode_slots, dtype=np.int64), prompt_slots])
