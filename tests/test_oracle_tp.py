"""The tensor-parallel partition of the dense block, stated on the CPU with the
oracle's own q4 arithmetic: column-split projections (q/k/v, gate/up) give
the rows of the full output, and the row-split projections (o, down) summed
over ranks -- the allreduce -- give the full output.  The weights of each
rank's slice come from the full tensor's synthesis, as on the device."""
import numpy as np

from oracle import oracle as O


def slice_cols(wq, s, b, c0, c1):
    return (np.ascontiguousarray(wq[:, c0 // 8:c1 // 8]), np.ascontiguousarray(s[:, c0 // 64:c1 // 64]),
            np.ascontiguousarray(b[:, c0 // 64:c1 // 64]))


def test_row_split_partials_sum_to_the_full_projection():
    N, K, T, M = 256, 1024, 4, 6
    wq, s, b = O.q4_synth(5, 77, 0.02, N, K)
    x = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
    full = O.q4_linear(wq, s, b, x)
    kl = K // T
    parts = [O.q4_linear(*slice_cols(wq, s, b, r * kl, (r + 1) * kl), np.ascontiguousarray(x[:, r * kl:(r + 1) * kl]))
             for r in range(T)]
    np.testing.assert_allclose(sum(parts), full, rtol=1e-5, atol=1e-5)


def test_column_split_rows_are_the_full_projection():
    N, K, T, M = 512, 256, 2, 5
    wq, s, b = O.q4_synth(5, 78, 0.02, N, K)
    x = np.random.default_rng(2).standard_normal((M, K)).astype(np.float32)
    full = O.q4_linear(wq, s, b, x)
    nl = N // T
    for r in range(T):
        part = O.q4_linear(wq[r * nl:(r + 1) * nl], s[r * nl:(r + 1) * nl], b[r * nl:(r + 1) * nl], x)
        np.testing.assert_array_equal(part, full[:, r * nl:(r + 1) * nl])
