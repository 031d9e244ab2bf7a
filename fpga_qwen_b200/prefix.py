"""Canonical 512-token prefix reuse: the adapter policy, with device block copies.

Policy (tampajohn/fpga-qwen tools/native_cpu_chat.py:189-221, engine/INTERFACE.md:151-168):

* reuse = floor(min(common prefix, canonical reusable tokens, len(request) - 1) / 512) * 512;
* only complete 512-token prefill chunks are canonical — decoded or verified KV and a
  partial prefill tail are never promoted (``canonical = len(prompt) // 512 * 512`` after a
  prefill, :221);
* at least one prompt token is always recomputed, and the whole remaining suffix is
  prefilled after the retained prefix.

The reference retains the prefix in place (``rewind``). Here a :class:`PrefixCache`
remembers which sequence slot holds which canonical token prefix; a new request either
rewinds its own slot or receives the prefix from another slot through
``qa_copy_prefix`` (a device block copy of 114,688 bytes per position), then recomputes
the tail.
"""
from __future__ import annotations

from dataclasses import dataclass, field

CHUNK = 512


def common_prefix(a, b) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def reuse_length(cached_ids, canonical_reusable: int, request_ids) -> int:
    """The adapter's reuse rule, native_cpu_chat.py:199-204."""
    if not request_ids:
        return 0
    common = common_prefix(cached_ids, request_ids)
    return (min(common, canonical_reusable, len(request_ids) - 1) // CHUNK) * CHUNK


def canonical_after_prefill(prompt_len: int) -> int:
    """Reusable length recorded after a full prefill, native_cpu_chat.py:221."""
    return (prompt_len // CHUNK) * CHUNK


@dataclass
class SlotState:
    ids: list = field(default_factory=list)
    canonical: int = 0


@dataclass
class Plan:
    slot: int            # slot that will serve the request
    source: int | None   # slot the prefix is copied from (None: rewind in place or fresh)
    reuse: int           # retained prefix length (multiple of 512)
    tail: int            # rows to prefill


class PrefixCache:
    """Tracks canonical prefixes held by sequence slots and plans each request."""

    def __init__(self, slots: int):
        self.slots = [SlotState() for _ in range(slots)]

    def plan(self, target: int, request_ids) -> Plan:
        best, best_slot = 0, None
        for i, s in enumerate(self.slots):
            r = reuse_length(s.ids, s.canonical, request_ids)
            if r > best or (r == best and r > 0 and i == target):
                best, best_slot = r, i
        if best == 0:
            return Plan(target, None, 0, len(request_ids))
        return Plan(target, None if best_slot == target else best_slot, best, len(request_ids) - best)

    def apply(self, ctx, plan: Plan):
        """Performs the device side of a plan: rewind in place, copy from another slot, or reset."""
        if plan.reuse == 0:
            ctx.reset(plan.slot)
        elif plan.source is None:
            ctx.truncate(plan.slot, plan.reuse)
        else:
            ctx.copy_prefix(plan.source, plan.slot, plan.reuse)

    def record_prefill(self, slot: int, request_ids):
        self.slots[slot] = SlotState(list(request_ids), canonical_after_prefill(len(request_ids)))

    def record_decode(self, slot: int, token: int):
        # Decoded KV extends the sequence but is never canonical (INTERFACE.md:110-111).
        self.slots[slot].ids.append(token)
