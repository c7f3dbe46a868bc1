"""The corpus batcher (src/libs/data/Corpus.cpp:25-107): the oracle's restatement pinned against
the reference compiled from its sources and its own test's known answers; (GPU) the device
batcher against the oracle, bit-exact."""
import numpy as np
import pytest

from oracle import ref as R
from oracle import veda_oracle as O

CASES = [(200, 0.0, 12345, 4, 8), (10, 0.2, 7, 2, 3), (1000, 0.25, 999, 4, 16), (500, 0.0, 0, 3, 10),
         (5000, 0.1, 2**63 + 11, 7, 33)]


def _ids(n, r=None):
    if r is None:
        return np.arange(n, dtype=np.int64)
    return r.integers(0, 151936, n).astype(np.int64)


def test_oracle_known_answers():
    # CorpusTest.cpp: boundaries, shifted targets, contiguous windows, windows inside the split
    assert O.Corpus(_ids(10) + 97, 0.2, 7).boundary == 8
    assert O.Corpus(_ids(1000), 0.25, 999).boundary == 750
    c = O.Corpus(_ids(200), 0.0, 12345)
    x, y = c.next_batch(4, 8)
    assert np.array_equal(y, x + 1) and np.all(np.diff(x, axis=1) == 1)
    c = O.Corpus(_ids(10) + 97, 0.2, 7)
    for _ in range(50):
        x, _ = c.next_batch(2, 3)
        assert np.all((x[:, 0] >= 97) & (x[:, 0] <= 101))
    with pytest.raises(ValueError):
        O.Corpus(_ids(10), 1.5, 1)
    with pytest.raises(ValueError):
        O.Corpus(_ids(10), 0.5, 1).next_batch(1, 5, "validation")


@pytest.mark.skipif(not R.available(), reason="reference not built")
@pytest.mark.parametrize("n,frac,seed,B,T", CASES)
def test_oracle_matches_reference(n, frac, seed, B, T):
    ids = _ids(n, np.random.default_rng(n))
    a, b = O.Corpus(ids, frac, seed), R.RefCorpus(ids, frac, seed)
    assert a.boundary == b.boundary
    for k in range(20):
        split = "validation" if (k % 3 == 2 and frac > 0 and n * frac > T + 1) else "train"
        xa, ya = a.next_batch(B, T, split)
        xb, yb = b.next_batch(B, T, split)
        assert np.array_equal(xa, xb) and np.array_equal(ya, yb), (k, split)


@pytest.mark.gpu
@pytest.mark.parametrize("n,frac,seed,B,T", CASES + [(2_000_000, 0.05, 3, 4, 2048)])
def test_device_batches_match_oracle(cuda, n, frac, seed, B, T):
    import torch
    from veda_b200 import train_abi as TA
    ids = _ids(n, np.random.default_rng(n))
    ref = O.Corpus(ids, frac, seed)
    dev = TA.Corpus(ids, frac, seed)
    assert dev.boundary == ref.boundary
    x = torch.empty(B * T, dtype=torch.int64, device="cuda")
    y = torch.empty_like(x)
    for k in range(12):
        split = "validation" if (k % 3 == 2 and frac > 0 and n * frac > T + 1) else "train"
        dev.next_batch(B, T, split, x.data_ptr(), y.data_ptr())
        xr, yr = ref.next_batch(B, T, split)
        torch.cuda.synchronize()
        assert np.array_equal(x.cpu().numpy().reshape(B, T), xr), (k, split)
        assert np.array_equal(y.cpu().numpy().reshape(B, T), yr), (k, split)
    # a split too short for the window raises and draws nothing
    if frac > 0:
        with pytest.raises(ValueError):
            dev.next_batch(1, int(n * frac) + 5, "validation", x.data_ptr(), y.data_ptr())
        dev.next_batch(B, T, "train", x.data_ptr(), y.data_ptr())
        xr, _ = ref.next_batch(B, T, "train")
        torch.cuda.synchronize()
        assert np.array_equal(x.cpu().numpy().reshape(B, T), xr)
    dev.close()
