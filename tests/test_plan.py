"""Host-side planning of the screens (metal-flat_b200/csrc/cuda/plan.h), on CPU.

plan.h decides how the database tiles are cut into chunks (work units = query
tile x chunk) and, for k beyond the list path, the floor-estimate plan.  These
tests compile a small probe against the header with g++ and check the plans'
invariants, and that the shapes the GPU tests rely on take the intended route.
"""
import itertools
import math
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "metal-flat_b200", "csrc", "cuda")
SMS = 148
GB = 1 << 30
BN = 256
BM = 128
FIELDS = ("prepass", "two_stage", "lists", "stride_a", "sample_a", "stride_b", "sample_b",
          "chunks_a", "tpc_a", "r_stat", "r_guess", "cap", "batch")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path_factory.mktemp("plan") / "plan_probe")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", INC,
                    os.path.join(ROOT, "tests", "plan_probe.cpp"), "-o", exe], check=True)

    def run(lines):
        out = subprocess.run([exe], input="\n".join(lines) + "\n", capture_output=True, text=True,
                             check=True).stdout.split("\n")
        return [list(map(int, o.split())) for o in out[:len(lines)]]
    return run


def large(probe, cases):
    res = probe(["large %d %d %d %d %d %d %d %d" % c for c in cases])
    return [dict(zip(FIELDS, r)) for r in res]


def test_chunks_cover_the_tiles(probe):
    cases = list(itertools.product([1, 3, 16, 79, 128], [1, 2, 7, 100, 391, 3907, 39063],
                                   [SMS, 8], [1, 16, 128, 256], [1, 5, 300]))
    res = probe(["chunks %d %d %d %d %d" % c for c in cases])
    for (nq, nt, sms, maxc, minc), (nc, tpc) in zip(cases, res):
        assert nc >= 1 and tpc >= 1
        assert nc * tpc >= nt and (nc - 1) * tpc < nt, (nq, nt, nc, tpc)
        if minc <= min(maxc, nt):
            assert nc <= min(maxc, nt)
            # at least `min_chunks` slices were asked for: no chunk is longer
            assert tpc <= -(-nt // minc)


def _span(nq, nt, slots, s):
    """Tiles the busiest slot streams when the tiles are cut into s chunks."""
    tpc = -(-nt // s)
    sc = -(-nt // tpc)
    return -(-(nq * sc) // slots) * tpc


def test_chunks_take_the_shortest_critical_path(probe):
    """The plan's critical path (waves x tiles per chunk) is within 1 % of the
    shortest over the chunk counts it may use, with the fewest such chunks; the
    config-3 pair plan is 11 chunks of 3,552 tiles (440 pair units: the last of
    six waves fills 70 of 74 slots) rather than 9 (360 units, 4.86 waves)."""
    cases = list(itertools.product([1, 4, 40, 79, 256, 39063], [1, 7, 256, 391, 3907, 39063],
                                   [SMS, SMS // 2], [16, 64, 128]))
    res = probe(["chunks %d %d %d %d 1" % c for c in cases])
    for (nq, nt, sms, maxc), (nc, tpc) in zip(cases, res):
        smax = min(maxc, nt, 1 + 4 * sms)
        best = min(_span(nq, nt, sms, s) for s in range(1, smax + 1))
        got = -(-(nq * nc) // sms) * tpc
        assert got * 100 <= best * 101, (nq, nt, sms, maxc, nc, tpc)
        fewer = [s for s in range(1, smax + 1) if _span(nq, nt, sms, s) * 100 <= best * 101]
        assert nc == -(-nt // (-(-nt // fewer[0]))), (nq, nt, sms, maxc, nc, fewer[0])
    (p,) = probe(["chunks 40 39063 74 128 1"])
    assert p == [11, 3552]


def test_buffer_chunks_fit_in_l2_budget(probe):
    cases = list(itertools.product([1, 16, 64, 128], [1, 977, 7813, 31250, 390625],
                                   [BN * 128 * 2, BN * 128 * 8, BN * 768 * 2, BN * 960 * 8]))
    res = probe(["buffer %d %d %d %d" % (nq, nt, SMS, tb) for nq, nt, tb in cases])
    for (nq, nt, tb), (nc, tpc) in zip(cases, res):
        assert nc * tpc >= nt and (nc - 1) * tpc < nt
        assert tpc <= max(16, (8 << 20) // tb), (nq, nt, tb, tpc)


def test_large_plan_invariants(probe):
    cases = []
    for n in [1, 1000, 32768, 32769, 60_000, 150_000, 200_003, 1_000_000, 2_000_000,
              3_000_000, 5_000_000, 8_000_000, 17_000_000, 20_000_000, 100_000_000]:
        for k, m in [(22, 30), (100, 10_000), (300, 17), (1024, 16_384), (1024, 5)]:
            cases.append((n, k, m, 32, 2 * k, 2, SMS, 16 * GB))      # fp32 exact path
            cases.append((n, k, m, 16, k, 2, SMS, 16 * GB))          # 16-bit buffer path
            cases.append((n, k, m, 16, k, 2, SMS, 1 * GB))
    for c, p in zip(cases, large(probe, cases)):
        n, k, m, kp1, want, lpc, sms, budget = c
        n_tiles = -(-n // BN)
        n_round = -(-n // 256) * 256
        assert 1 <= p["batch"] <= m
        assert p["batch"] == m or p["batch"] >= BM
        assert p["cap"] <= n_round and (p["cap"] % 256 == 0 or p["cap"] == n_round)
        if p["batch"] > BM:       # a batch's candidate buffers stay within the budget
            assert p["batch"] * (p["cap"] * 8 + 64) <= budget
        if n <= 32768:
            assert not p["prepass"] and p["cap"] == n_round
            continue
        if not p["prepass"]:       # too few tiles to sample: every row is buffered
            assert p["cap"] == n_round
            continue
        lists = p["lists"]
        assert lists * lpc * kp1 >= min(2 * want, 4096 - kp1 * lpc + 1)
        assert p["sample_b"] == -(-n_tiles // p["stride_b"]) >= lists
        # >= `lists` chunks, unless one tile fewer per chunk would overflow the
        # floor select's fan-in; either way the union holds >= want scores
        max_a = max(lists, 4096 // (kp1 * lpc))
        finer = -(-p["sample_a"] // (p["tpc_a"] - 1)) if p["tpc_a"] > 1 else None
        assert p["chunks_a"] >= lists or (finer is not None and finer > max_a)
        assert p["chunks_a"] <= max_a
        assert p["chunks_a"] * lpc * kp1 >= want
        assert p["chunks_a"] * p["tpc_a"] >= p["sample_a"] > (p["chunks_a"] - 1) * p["tpc_a"]
        # the floor select takes the union of the stage-A lists
        assert p["chunks_a"] * lpc * kp1 <= max(4096, lists * lpc * kp1)
        assert p["cap"] >= min(4 * want * p["stride_b"], n_round) or p["cap"] == n_round
        if p["two_stage"]:
            assert p["stride_b"] == 16 and p["stride_a"] in (64, 128, 256)
            assert p["sample_a"] == -(-n_tiles // p["stride_a"]) >= 2 * lists
            # the sparsest stride that still gives every list two tiles
            if p["stride_a"] < 256:
                assert -(-n_tiles // (2 * p["stride_a"])) < 2 * lists
            mean = want / 16
            r = math.ceil(mean + 6 * math.sqrt(mean)) + 1
            assert p["r_stat"] == (r if r < want else 0)
            mean_a = want * 16 / p["stride_a"]
            ra = math.ceil(mean_a + 6 * math.sqrt(mean_a)) + 1
            assert p["r_guess"] == (ra if ra < want else 0)
        else:
            assert p["stride_a"] == p["stride_b"] and p["r_stat"] == 0 and p["r_guess"] == 0
            if p["stride_b"] == 16:
                assert -(-n_tiles // 64) < 2 * lists


@pytest.mark.parametrize("case,route", [
    # config 5 (bf16, 100M rows, Q = 16,384, k = 1024): stage A over every 256th tile
    ((100_000_000, 1024, 16_384, 16, 1024, 2), ("two", 256)),
    # the 8M-row and 3M-row 16-bit cases: denser stage-A samples
    ((8_000_000, 1024, 16_384, 16, 1024, 2), ("two", 128)),
    ((3_000_000, 1024, 6, 16, 1024, 2), ("two", 64)),
    # fp32 k = 1024 (two stage-A lists per chunk): 17M and 10M rows (1/256),
    # 5M rows (1/128)
    ((17_000_000, 1024, 6, 32, 2048, 2), ("two", 256)),
    ((10_000_000, 1024, 2048, 32, 2048, 2), ("two", 256)),
    ((5_000_000, 1024, 5, 32, 2048, 2), ("two", 128)),
    # exact-path shapes with a single-stage pre-pass or none (k = 1024 on 586
    # tiles: the stride halves until the 64 chunks of 2 lists fit), and a
    # small k that gets both stages
    ((150_000, 1024, 33, 32, 2048, 2), ("one", 4)),
    ((150_000, 64, 40, 32, 128, 2), ("two", 64)),
    ((2_000_000, 100, 2, 32, 200, 2), ("two", 256)),
    ((3000, 300, 17, 32, 600, 2), ("none", 0)),
    # config 2 (fp16, 1M rows, k = 100): two-stage at 1/256
    ((1_000_000, 100, 10_000, 16, 100, 2), ("two", 256)),
])
def test_routes_of_the_tested_shapes(probe, case, route):
    (p,) = large(probe, [case + (SMS, 16 * GB)])
    kind, stride = route
    if kind == "none":
        assert not p["prepass"]
    elif kind == "one":
        assert p["prepass"] and not p["two_stage"] and p["stride_a"] == stride
    else:
        assert p["two_stage"] and p["stride_a"] == stride and p["stride_b"] == 16


def test_config5_batch_and_ranks(probe):
    """Config 5 runs as one query batch; the statistical floor admits about
    r_stat * 16 rows per query instead of want * 16."""
    (p,) = large(probe, [(100_000_000, 1024, 16_384, 16, 1024, 2, SMS, 16 * GB)])
    assert p["batch"] == 16_384
    assert p["cap"] == 4 * 1024 * 16
    assert p["r_stat"] == 113 and p["r_guess"] == 113
