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
the tail. :class:`BlockPrefixCache` keeps canonical chunks in a device block pool
(``qa_block_pool``) so that they outlive the slots that computed them: a tree of 512-token
chunks keyed by the whole token prefix, evicted leaf first in least-recently-used order.
"""
from __future__ import annotations

import hashlib
import struct
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


@dataclass(eq=False)          # identity: chains and the eviction guard compare objects
class _Block:
    block: int           # pool block holding the chunk
    chunk: int           # chunk index: rows [512*chunk, 512*chunk + 512)
    tokens: tuple        # the chunk's token ids (checked on every match)
    parent: "_Block | None"
    children: int = 0
    last_use: int = 0


class BlockPrefixCache:
    """Cross-session canonical prefix cache over the device block pool.

    Chunk i of a token sequence is keyed by a digest of tokens [0, 512*(i+1)) and stored in
    one pool block (``qa_block_save``). A request receives the longest chain of cached
    chunks that the adapter's rule allows (a multiple of 512, at least one token left to
    recompute) through ``qa_block_load``, then prefills the rest. Only chunks of a prompt's
    prefill are saved: decoded or verified KV is never canonical (INTERFACE.md:110-111,
    native_cpu_chat.py:221). A full pool evicts the least recently used chunk that no cached
    chunk extends, so every cached chunk's ancestors stay cached.
    """

    def __init__(self, ctx, n_blocks: int):
        self.ctx = ctx
        ctx.block_pool(n_blocks)
        self.free = list(range(n_blocks - 1, -1, -1))
        self.entries: dict[bytes, _Block] = {}
        self.clock = 0

    @staticmethod
    def digests(ids, n_chunks: int) -> list:
        h = hashlib.sha256()
        out = []
        for i in range(n_chunks):
            chunk = ids[i * CHUNK:(i + 1) * CHUNK]
            h.update(struct.pack(f"<{len(chunk)}q", *chunk))
            out.append(h.copy().digest())
        return out

    def _touch(self, e: _Block):
        self.clock += 1
        e.last_use = self.clock

    def match(self, request_ids) -> list:
        """Cached chunks that a request may reuse, in order (possibly empty)."""
        if not request_ids:
            return []
        limit = (len(request_ids) - 1) // CHUNK          # at least one prompt token is recomputed
        chain, parent = [], None
        for i, d in enumerate(self.digests(request_ids, limit)):
            e = self.entries.get(d)
            if e is None or e.parent is not parent or e.tokens != tuple(request_ids[i * CHUNK:(i + 1) * CHUNK]):
                break
            chain.append(e)
            parent = e
        return chain

    def load(self, seq: int, request_ids) -> int:
        """Resets slot seq and loads the request's reusable cached prefix; returns its length
        (the caller prefills tokens [length, len(request_ids)) next)."""
        chain = self.match(request_ids)
        self.ctx.reset(seq)
        for e in chain:
            self.ctx.block_load(seq, e.chunk, e.block)
            self._touch(e)
        return len(chain) * CHUNK

    def _allocate(self, keep) -> int | None:
        if self.free:
            return self.free.pop()
        kept = {id(e) for e in keep}
        leaves = [e for e in self.entries.values() if e.children == 0 and id(e) not in kept]
        if not leaves:
            return None
        victim = min(leaves, key=lambda e: e.last_use)
        for d, e in list(self.entries.items()):
            if e is victim:
                del self.entries[d]
                break
        if victim.parent is not None:
            victim.parent.children -= 1
        return victim.block

    def save(self, seq: int, prompt_ids) -> int:
        """After the prefill of prompt_ids into slot seq (rows committed), caches its canonical
        chunks that are not cached yet; returns how many chunks of the prompt are cached."""
        n = canonical_after_prefill(len(prompt_ids)) // CHUNK
        parent, chain = None, []
        for i, d in enumerate(self.digests(prompt_ids, n)):
            e = self.entries.get(d)
            if e is None:
                block = self._allocate(chain)
                if block is None:
                    break
                try:
                    self.ctx.block_save(seq, i, block)
                except Exception:
                    self.free.append(block)      # the block holds nothing cached any more
                    raise
                e = _Block(block, i, tuple(prompt_ids[i * CHUNK:(i + 1) * CHUNK]), parent)
                self.entries[d] = e
                if parent is not None:
                    parent.children += 1
            self._touch(e)
            chain.append(e)
            parent = e
        return len(chain)
