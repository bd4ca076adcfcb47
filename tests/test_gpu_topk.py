"""qwen_row_topk (the device top-k of the batched decode step) against a numpy
selection of the same rows: the k best entries of each row by value, ties to
the smaller column, NaN below every number, -0 equal to +0.  The kernel returns
its k entries in column order; both sides are compared as sorted lists, ids
exactly and values bit for bit (up to the sign of zero)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _expected(row, k):
    n = row.size
    nan = np.isnan(row)
    v = np.where(nan, 0.0, row).astype(np.float64)
    v = np.where(v == 0.0, 0.0, v)
    return np.lexsort((np.arange(n), -v, nan))[:k]


def _run(qb, rows_np, k, ld=None):
    import torch
    rows, n = rows_np.shape
    ld = ld or n
    buf = np.full((rows, ld), 7.0, dtype=np.float32)      # columns past n must not be read
    buf[:, :n] = rows_np
    L = torch.from_numpy(buf).cuda()
    V = torch.empty(rows, k, dtype=torch.float32, device="cuda")
    I = torch.empty(rows, k, dtype=torch.int32, device="cuda")
    qb.row_topk(L.data_ptr(), rows, n, ld, k, V.data_ptr(), I.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return V.cpu().numpy(), I.cpu().numpy()


def _check(rows_np, V, I, k):
    for r in range(rows_np.shape[0]):
        ids = I[r]
        assert np.all(np.diff(ids) > 0), "not in column order"
        exp = _expected(rows_np[r], k)
        got_sorted = ids[_expected(rows_np[r][ids], k)]           # the kernel's set, ordered the same way
        np.testing.assert_array_equal(got_sorted, exp)
        np.testing.assert_array_equal(V[r], np.where(rows_np[r][ids] == 0, 0.0, rows_np[r][ids]))


@pytest.mark.parametrize("k", [1, 2, 20, 40, 64])
def test_topk_vocab_rows(qb, k):
    rng = np.random.default_rng(100 + k)
    x = (rng.standard_normal((8, 151936)) * 3).astype(np.float32)
    V, I = _run(qb, x, k)
    _check(x, V, I, k)


@pytest.mark.parametrize("n,k", [(1, 1), (64, 64), (100, 20), (512, 64), (513, 20), (1000, 64), (5000, 20), (26 * 512 + 7, 20)])
def test_topk_ragged_lengths(qb, n, k):
    rng = np.random.default_rng(n * 131 + k)
    x = rng.standard_normal((3, n)).astype(np.float32)
    V, I = _run(qb, x, k, ld=n + 12)
    _check(x, V, I, k)


@pytest.mark.parametrize("k", [1, 20, 64])
def test_topk_ties_and_specials(qb, k):
    """Few distinct values (ties across the k boundary in every group and level),
    -inf, NaN and both zeros."""
    rng = np.random.default_rng(7 + k)
    x = rng.integers(-3, 4, size=(4, 151936)).astype(np.float32)
    x[0, rng.integers(0, 151936, 5000)] = -np.inf
    x[1, rng.integers(0, 151936, 5000)] = np.nan
    x[2] = np.where(x[2] == 0, -0.0, x[2]).astype(np.float32)
    x[3, :] = -np.inf
    x[3, rng.integers(0, 151936, 10)] = 1.5
    V, I = _run(qb, x, k)
    _check(x, V, I, k)


def test_topk_all_equal_row_takes_the_first_columns(qb):
    x = np.full((2, 151936), 0.25, dtype=np.float32)
    V, I = _run(qb, x, 64)
    np.testing.assert_array_equal(I, np.tile(np.arange(64, dtype=np.int32), (2, 1)))


def test_topk_many_rows(qb):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((128, 151936)).astype(np.float32)
    V, I = _run(qb, x, 20)
    _check(x, V, I, 20)


def test_topk_errors(qb):
    with pytest.raises(qb.QwenError):
        qb.row_topk(0, 1, 10, 10, 1, 0, 0)
    import torch
    L = torch.zeros(1, 16, device="cuda")
    V = torch.empty(65, device="cuda")
    I = torch.empty(65, dtype=torch.int32, device="cuda")
    for rows, n, ld, k in [(0, 16, 16, 1), (1, 16, 8, 1), (1, 16, 16, 0), (1, 16, 16, 65)]:
        with pytest.raises(qb.QwenError):
            qb.row_topk(L.data_ptr(), rows, n, ld, k, V.data_ptr(), I.data_ptr())
