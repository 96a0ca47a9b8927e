"""The C ABI library loads, exports every symbol include/*.h declares, and
its host-only entry points behave like the reference (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(mvr_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from ir_multivector_retrieval_b200 import _lib

    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 18
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_header(lib):
    from ir_multivector_retrieval_b200 import _lib

    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_status_names_match_zig_errors(lib):
    from ir_multivector_retrieval_b200._lib import STATUS_NAMES

    for code, name in STATUS_NAMES.items():
        assert lib.mvr_status_name(code).decode() == name


def test_decode_on_host(lib):
    from ir_multivector_retrieval_b200 import pq

    rng = np.random.default_rng(1)
    cb = rng.standard_normal(16 * 256 * 4).astype(np.float32)
    codes = rng.integers(0, 256, size=(7, 16), dtype=np.uint8)
    p = pq.PQ(dim=64, sub_dim=4, codebooks=cb, pq_m=16)
    dec = p.decode(codes)
    want = cb.reshape(16, 256, 4)[np.arange(16)[None, :], codes].reshape(7, 64)
    assert np.array_equal(dec, want)


def test_allocate_budgets_matches_reference_kats(lib):
    from ir_multivector_retrieval_b200 import tac

    # src/tac/tac.zig:1041-1086
    k = tac.allocate_budgets([0, 2, 4, 20, 20, 20], [0, 0, 0, 1.0, 2.0, 3.0], 18,
                             tac.ClusteringParams(kappa_total=18, seed=0, mu=3, tau=5, epsilon=4, theta=1))
    assert list(k) == [0, 1, 2, 4, 4, 7]
    with pytest.raises(Exception) as e:
        tac.allocate_budgets([1, 1, 4], [0, 0, 0], 3, tac.ClusteringParams(kappa_total=3, seed=0, mu=3, tau=5))
    assert e.value.name == "BudgetTooSmall"


def test_allocate_budgets_matches_oracle_on_random_vocab(lib, orc):
    from ir_multivector_retrieval_b200 import tac

    rng = np.random.default_rng(5)
    freqs = (rng.zipf(1.3, size=3000) * 3).astype(np.uint32)
    freqs[rng.random(3000) < 0.1] = 0
    spreads = rng.random(3000).astype(np.float32)
    tail = int(((freqs > 0) & (freqs < 128)).sum() + 2 * ((freqs >= 128) & (freqs < 256)).sum())
    active = int((freqs >= 256).sum())
    kt = tail + 4 * active + 500
    want = orc.tac_allocate_budgets(freqs, spreads, kt)
    got = tac.allocate_budgets(freqs, spreads, kt, tac.ClusteringParams(kappa_total=kt, seed=0))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("seed", range(12))
def test_allocate_budgets_reconcile_paths_match_oracle(lib, orc, seed):
    """Surplus, deficit, degraded-tail and failing budgets: the host phase 4
    (one pass in remainder order) against the oracle's one-unit rounds."""
    from ir_multivector_retrieval_b200 import tac

    rng = np.random.default_rng(100 + seed)
    n = int(rng.integers(5, 400))
    freqs = (np.minimum(rng.zipf(1.2, size=n), 400) * int(rng.integers(1, 40))).astype(np.uint32)
    freqs[rng.random(n) < 0.1] = 0
    spreads = rng.random(n).astype(np.float32)
    spreads[rng.random(n) < 0.2] = 0.0
    spreads[rng.random(n) < 0.1] = spreads[0]  # equal remainders
    mu, tau, eps, theta = [(128, 256, 4, 39), (3, 40, 2, 10), (8, 64, 1, 4)][seed % 3]
    tail = int(((freqs > 0) & (freqs < mu)).sum() + 2 * ((freqs >= mu) & (freqs < tau)).sum())
    cap = int(sum(f // theta for f in freqs if f >= tau))
    for kt in {max(1, tail // 2), max(1, tail - 3), tail + 1, tail + cap // 3, tail + cap, tail + cap + 7}:
        p = tac.ClusteringParams(kappa_total=kt, seed=0, mu=mu, tau=tau, epsilon=eps, theta=theta)
        try:
            want = orc.tac_allocate_budgets(freqs, spreads, kt, mu, tau, eps, theta)
        except Exception as e:
            with pytest.raises(Exception) as g:
                tac.allocate_budgets(freqs, spreads, kt, p)
            assert g.value.code == e.code
            continue
        got = tac.allocate_budgets(freqs, spreads, kt, p)
        assert np.array_equal(got, want), (kt, mu, tau, eps, theta)


def test_no_gpu_fails_loudly_or_creates_context(lib):
    h = C.c_void_p()
    st = lib.mvr_ctx_create(0, C.byref(h))
    if st == 0:
        lib.mvr_ctx_destroy(h)
    else:
        assert lib.mvr_status_name(st).decode() in ("NoDevice", "CudaError")


def test_crc32_matches_the_standard(lib):
    import zlib

    from ir_multivector_retrieval_b200 import storage

    assert storage.crc32(b"123456789") == 0xCBF43926  # the published CRC-32 check value
    rng = np.random.default_rng(0)
    for n in (0, 1, 7, 8, 9, 4097):
        d = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        assert storage.crc32(d) == zlib.crc32(d)
        assert storage.crc32(d[n // 2:], storage.crc32(d[:n // 2])) == zlib.crc32(d)


def test_doc_layout_size_matches_oracle(lib, orc):
    from ir_multivector_retrieval_b200 import storage

    rng = np.random.default_rng(3)
    for m in (16, 32, 3):
        n_d = rng.integers(0, 9, size=50)
        off = np.concatenate([[0], np.cumsum(n_d)]).astype(np.uint64)
        n = int(off[-1])
        b = orc.write_doc_layouts(off, rng.integers(0, 1000, size=n), rng.integers(0, 256, size=n * m), m)
        assert storage.doc_layouts_bytes(off, m) == len(b)
