"""Canonical prefix-reuse policy (tools/native_cpu_chat.py:189-221) — host logic, no GPU."""
from fpga_qwen_b200.prefix import PrefixCache, canonical_after_prefill, reuse_length


class FakeCtx:
    def __init__(self):
        self.calls = []

    def reset(self, s):
        self.calls.append(("reset", s))

    def truncate(self, s, p):
        self.calls.append(("truncate", s, p))

    def copy_prefix(self, a, b, n):
        self.calls.append(("copy", a, b, n))


def test_reuse_rule_matches_adapter():
    ids = list(range(2000))
    # full canonical chunks only, at least one token recomputed, rounded down to 512
    assert reuse_length(ids, 1536, ids[:1537]) == 1536
    assert reuse_length(ids, 1536, ids[:1536]) == 1024        # keep >= 1 token to recompute
    assert reuse_length(ids, 1536, ids[:1025]) == 1024
    assert reuse_length(ids, 1536, ids[:1024]) == 512
    assert reuse_length(ids, 1024, ids) == 1024                # capped by canonical end
    assert reuse_length(ids, 1536, ids[:511] + [-1] + ids[512:]) == 0   # edit at 511
    assert reuse_length(ids, 1536, ids[:512] + [-1] + ids[513:]) == 512  # edit at 512
    assert reuse_length(ids, 1536, ids[:1024] + [-1]) == 1024             # edit at 1024
    assert reuse_length([], 0, ids) == 0
    assert reuse_length(ids, 1536, []) == 0


def test_canonical_end_after_prefill():
    for n, c in [(1, 0), (511, 0), (512, 512), (513, 512), (1024, 1024), (1025, 1024), (3968, 3584)]:
        assert canonical_after_prefill(n) == c


def test_plan_rewinds_in_place_or_copies_between_slots():
    cache = PrefixCache(3)
    a = list(range(1024))
    cache.record_prefill(0, a)
    b = a[:512] + [9] * 512
    ctx = FakeCtx()
    plan = cache.plan(1, b)                 # another slot holds the prefix -> device copy
    assert (plan.slot, plan.source, plan.reuse, plan.tail) == (1, 0, 512, 512)
    cache.apply(ctx, plan)
    assert ctx.calls == [("copy", 0, 1, 512)]
    plan = cache.plan(0, a + [5])           # same slot -> rewind in place
    assert (plan.source, plan.reuse) == (None, 1024)
    cache.apply(ctx, plan)
    assert ctx.calls[-1] == ("truncate", 0, 1024)
    plan = cache.plan(2, [7] * 600)         # nothing shared -> fresh
    cache.apply(ctx, plan)
    assert plan.reuse == 0 and ctx.calls[-1] == ("reset", 2)


def test_decoded_tokens_never_become_canonical():
    cache = PrefixCache(1)
    cache.record_prefill(0, list(range(600)))
    for t in range(600):
        cache.record_decode(0, t)
    assert cache.slots[0].canonical == 512
    assert cache.plan(0, cache.slots[0].ids + [1]).reuse == 512
