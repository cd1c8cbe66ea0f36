"""CPU: context tiers (Tiers, the host side of packs/dory/npu.cpp's buckets and NpuModel::fit, npu.cpp:181-198) over
a fake session whose grow checks what xtg_cuda_grow checks (a tier of a multiple of 64 that holds the positions).
The device move itself is tested on the GPU (tests/test_gpu_session.py)."""
import pytest


class FakeSession:
    def __init__(self, context):
        self.context = context
        self.n_past = 0
        self.grows = []

    def info(self):
        return {"context": self.context}

    def pos(self):
        return self.n_past

    def grow(self, ctx):
        assert ctx % 64 == 0 and ctx >= self.n_past, (ctx, self.n_past)
        self.context = ctx
        self.grows.append(ctx)

    def forward(self, tokens, want=2):
        assert self.n_past + len(tokens) <= self.context, "forward past the tier"
        self.n_past += len(tokens)
        return {}

    def rewind(self, n):
        self.n_past = min(self.n_past, n)


def test_fit_picks_smallest_tier_with_room(xtg):
    s = FakeSession(4096)
    t = xtg.Tiers(s, [4096, 8192, 32768])
    assert t.context == 32768
    t.forward([1] * 4000)
    assert s.grows == []
    t.forward([1] * 200)          # 4200 positions: up one tier
    assert s.grows == [8192] and s.context == 8192
    t.forward([1] * 10000)        # 14200: past 8192 into 32768
    assert s.grows == [8192, 32768]
    t.forward([1] * 8)
    assert s.grows == [8192, 32768]


def test_fit_moves_down_for_a_shorter_conversation(xtg):
    s = FakeSession(4096)
    t = xtg.Tiers(s, [4096, 8192, 32768])
    t.forward([1] * 20000)
    assert s.context == 32768
    s.rewind(100)                 # a new conversation shares 100 positions of prefix
    t.forward([1] * 50)
    assert s.grows == [32768, 4096] and s.context == 4096


def test_fit_never_drops_held_positions(xtg):
    """fit(need) with fewer needed positions than the session holds (a caller that rewinds later) keeps the tier,
    as npu.cpp:188 returns when pos exceeds the chosen bucket."""
    s = FakeSession(4096)
    t = xtg.Tiers(s, [4096, 8192])
    t.forward([1] * 6000)
    assert s.context == 8192
    t.fit(100)
    assert s.context == 8192 and s.grows == [8192]


def test_fit_context_full(xtg):
    s = FakeSession(4096)
    t = xtg.Tiers(s, [4096, 8192])
    with pytest.raises(xtg.XtgError, match="context full: 9000 positions"):
        t.forward([1] * 9000)
    assert s.grows == [] and s.n_past == 0


def test_single_tier_never_grows(xtg):
    s = FakeSession(4096)
    t = xtg.Tiers(s, [4096])
    t.forward([1] * 4096)
    assert s.grows == []


@pytest.mark.parametrize("tiers,needle", [([], "no context tiers"), ([4096, 4096], "list the tiers by context"),
                                          ([8192, 4096], "list the tiers by context"),
                                          ([8192, 16384], "the first tier 8192")])
def test_bad_tier_lists(xtg, tiers, needle):
    with pytest.raises(xtg.XtgError, match=needle):
        xtg.Tiers(FakeSession(4096), tiers)
