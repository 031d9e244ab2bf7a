"""Cross-session prefix cache over the device block pool — host logic, no GPU.

The fake context enforces the C ABI's preconditions (qa_block_save: committed rows;
qa_block_load: the sequence sits at the chunk's first position and the block was saved from
the same chunk index) and tracks which token each KV row holds, so a wrong plan shows up as
a row that does not belong to the request.
"""
import pytest

from fpga_qwen_b200.prefix import CHUNK, BlockPrefixCache


class PoolCtx:
    def __init__(self, slots, context=4096):
        self.rows = [[] for _ in range(slots)]      # token id behind each committed KV row
        self.pool = {}
        self.n_blocks = 0
        self.context = context
        self.loads = 0

    def block_pool(self, n):
        self.n_blocks, self.pool = n, {}

    def reset(self, s):
        self.rows[s] = []

    def prefill(self, s, ids):                      # append + commit of the tail
        self.rows[s] = self.rows[s] + list(ids)
        assert len(self.rows[s]) <= self.context

    def block_save(self, s, chunk, block):
        assert 0 <= block < self.n_blocks
        assert len(self.rows[s]) >= (chunk + 1) * CHUNK, "chunk not committed"
        self.pool[block] = (chunk, self.rows[s][chunk * CHUNK:(chunk + 1) * CHUNK])

    def block_load(self, s, chunk, block):
        saved_chunk, rows = self.pool[block]
        assert saved_chunk == chunk, "block loaded at another chunk index"
        assert len(self.rows[s]) == chunk * CHUNK, "sequence not at the chunk's first position"
        self.rows[s] = self.rows[s] + rows
        self.loads += 1


def serve(cache, ctx, slot, ids):
    """One request: load the cached prefix, prefill the rest, cache the canonical chunks."""
    reused = cache.load(slot, ids)
    ctx.prefill(slot, ids[reused:])
    assert ctx.rows[slot] == list(ids)             # every KV row belongs to this request
    cache.save(slot, ids)
    return reused


def toks(seed, n):
    return [(seed * 7919 + i * 104729) % 151_936 for i in range(n)]


def test_reuse_across_slots_and_sessions():
    ctx = PoolCtx(2)
    cache = BlockPrefixCache(ctx, 8)
    a = toks(1, 1300)
    assert serve(cache, ctx, 0, a) == 0            # nothing cached yet; chunks 0, 1 saved
    # the slot that computed the prefix is overwritten by an unrelated request ...
    assert serve(cache, ctx, 0, toks(2, 600)) == 0
    # ... and a later request sharing 1100 tokens still gets both canonical chunks
    b = a[:1100] + toks(3, 300)
    assert serve(cache, ctx, 1, b) == 1024
    # a request that is exactly the cached prefix keeps one token to recompute
    assert serve(cache, ctx, 1, a[:1024]) == 512
    # a divergence inside chunk 1 reuses chunk 0 only
    c = a[:700] + toks(4, 500)
    assert serve(cache, ctx, 0, c) == 512


def test_decoded_rows_and_partial_chunks_are_never_cached():
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 4)
    a = toks(5, 1000)
    serve(cache, ctx, 0, a)                         # 1 canonical chunk (1000 // 512)
    ctx.prefill(0, toks(6, 100))                    # decoded tokens extend the slot, not the cache
    assert len(cache.entries) == 1
    assert serve(cache, ctx, 0, a + toks(6, 100)) == 512


def test_full_pool_evicts_least_recent_leaf_and_keeps_ancestors():
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 3)
    a = toks(7, 3 * CHUNK + 1)                      # chunks a0 a1 a2 fill the pool
    assert serve(cache, ctx, 0, a) == 0
    assert len(cache.entries) == 3
    b = a[:CHUNK] + toks(8, CHUNK + 1)              # shares a0; b1 needs a block
    assert serve(cache, ctx, 0, b) == 512
    # the least recently used leaf (a2) went; a0 (an ancestor) and a1 stayed
    assert len(cache.entries) == 3
    assert [e.chunk for e in cache.match(a)] == [0, 1]
    assert [e.chunk for e in cache.match(b + [1])] == [0, 1]
    # every cached chunk's parent is cached
    cached = {id(e) for e in cache.entries.values()}
    assert all(e.parent is None or id(e.parent) in cached for e in cache.entries.values())


def test_chain_being_saved_is_never_evicted():
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 2)
    a = toks(9, 3 * CHUNK + 1)                      # three chunks, room for two
    serve(cache, ctx, 0, a)
    assert [e.chunk for e in cache.match(a)] == [0, 1]


def test_match_checks_tokens_not_only_digests():
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 2)
    a = toks(10, 2 * CHUNK)
    serve(cache, ctx, 0, a)
    # plant a corrupted entry: the digest of chunk 0 now points at other tokens
    entry = next(iter(cache.entries.values()))
    entry.tokens = tuple(toks(11, CHUNK))
    assert cache.match(a) == []


@pytest.mark.parametrize("n", [0, 1, 511, 512, 513])
def test_short_requests_reuse_nothing(n):
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 2)
    serve(cache, ctx, 0, toks(12, 2 * CHUNK))
    assert cache.load(0, toks(12, n)) == (512 if n == 513 else 0)


def test_failed_save_returns_its_block():
    ctx = PoolCtx(1)
    cache = BlockPrefixCache(ctx, 2)
    ids = toks(13, 2 * CHUNK + 1)
    ctx.prefill(0, ids[:CHUNK + 10])               # only chunk 0 is committed
    with pytest.raises(AssertionError):
        cache.save(0, ids)                          # chunk 1 is refused by the (fake) library
    assert len(cache.entries) == 1 and len(cache.free) == 1
    ctx.prefill(0, ids[CHUNK + 10:])
    assert cache.save(0, ids) == 2                  # the returned block serves chunk 1
