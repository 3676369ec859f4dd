"""BatchKVCache row operations on the device through the C ABI:
filter(keeping:) (BatchCache.swift:217-245) and the per-row form of trim
(BatchCache.swift:403-424), on the reference's table test double."""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mlxcat_b200 as M  # noqa: E402


def table_cache(rows=3):
    vocab = 16
    ctx = M.Context(M.ModelConfig.table(vocab))
    ctx.set_table([(t + 1) % vocab for t in range(vocab)])
    cache = M.BatchKVCache(ctx, rows, 64)
    for r, n in enumerate((5, 9, 2)[:rows]):
        cache.insert_row(r, list(range(1, n + 1)), 8, M.SamplingParameters())
    return ctx, cache


def test_filter_keeps_listed_rows_in_their_slots():
    ctx, cache = table_cache()
    before = cache.lengths()
    cache.filter([2, 0])
    assert list(cache.active()) == [1, 0, 1]
    after = cache.lengths()
    assert after[0] == before[0] and after[2] == before[2] and after[1] == 0
    cache.filter([])
    assert list(cache.active()) == [0, 0, 0]


def test_trim_row_rolls_back_one_row():
    ctx, cache = table_cache()
    before = cache.lengths()
    assert cache.trim_row(1, 4) == 4
    assert cache.trim_row(2, 10) == before[2]   # clipped at the row's length
    after = cache.lengths()
    assert after[0] == before[0] and after[1] == before[1] - 4 and after[2] == 0
