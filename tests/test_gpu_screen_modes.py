"""Both tensor-core screen modes against the oracle: single CTAs (M = 128 per
MMA) and CTA pairs (tcgen05 cta_group::2, M = 256 over two SMs, each SM
holding half of every database tile).  Pairs are the default for batches of
two or more query tiles; MFLAT_SCREEN_PAIR=0 at index creation selects single
CTAs.  Each case runs in both modes: fp32 exact ids (list path and large-k
buffer path, odd query-tile counts so a pair's second tile is empty) and
16-bit storage against the oracle on the rounded rows."""
import zlib

import numpy as np
import pytest
import torch

import mflat_b200 as M
import oracle as O

pytestmark = pytest.mark.gpu


def _index(monkeypatch, pair, dim, metric, storage="fp32"):
    monkeypatch.setenv("MFLAT_SCREEN_PAIR", pair)
    idx = M.FlatIndex(dim, metric, storage)          # read at creation
    monkeypatch.delenv("MFLAT_SCREEN_PAIR")
    return idx


FP32 = [  # n, dim, m, k: list path (k <= 21) and large-k buffer path
    (60_000, 128, 383, 10), (30_000, 64, 257, 21), (50_000, 128, 300, 100), (40_000, 200, 130, 40),
]


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("metric", ["l2", "ip"])
@pytest.mark.parametrize("case", FP32, ids=lambda c: "n%d_d%d_m%d_k%d" % c)
def test_fp32_exact_both_modes(monkeypatch, pair, metric, case):
    n, dim, m, k = case
    rng = np.random.default_rng(zlib.crc32(repr((metric,) + case).encode()))
    db = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((m, dim)).astype(np.float32)
    idx = _index(monkeypatch, pair, dim, metric)
    idx.add(db)
    ids, dist = idx.search(q, k)
    idx.close()
    ref_i, ref_d = O.flat_search_f64(db, q, k + 1, O.L2 if metric == "l2" else O.IP)
    assert O.exact_ids_match(ids, dist, ref_i, ref_d, rel=1e-6) == 0


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("k", [10, 200])
def test_bf16_both_modes(monkeypatch, pair, k):
    rng = np.random.default_rng(77 + k)
    db = rng.standard_normal((80_000, 128)).astype(np.float32)
    q = rng.standard_normal((300, 128)).astype(np.float32)
    idx = _index(monkeypatch, pair, 128, "l2", "bf16")
    idx.add(db)
    ids, dist = idx.search(q, k)
    idx.close()
    dbr = torch.from_numpy(db).to(torch.bfloat16).float().numpy()
    qr = torch.from_numpy(q).to(torch.bfloat16).float().numpy()
    ref_i, ref_d = O.flat_search_f64(dbr, qr, k + 1, O.L2)
    assert O.exact_ids_match(ids, dist, ref_i, ref_d, rel=1e-4) == 0
