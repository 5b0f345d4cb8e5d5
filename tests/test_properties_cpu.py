"""Property-based checks of the oracle on arbitrary inputs (hypothesis):
termination within the iteration cap, row-stochastic output, invariance to
row and column shifts of the logits, and the backward's zero row/column sums."""
import numpy as np
from hypothesis import given, settings, strategies as st
from hypothesis.extra.numpy import arrays

import oracle

finite = st.floats(min_value=-30, max_value=30, allow_nan=False, width=32)
any_float = st.floats(width=32, allow_nan=True, allow_infinity=True)


@settings(max_examples=60, deadline=None)
@given(arrays(np.float32, (8, 4, 4), elements=finite))
def test_rows_sum_to_one_and_cap(R):
    T, ev = oracle.birkhoff_proj_n4(R, 1e-6, return_evals=True, threads=1)
    assert np.all(ev <= 3 + 20 * 7)
    assert np.all(T >= 0)
    assert np.max(np.abs(T.astype(np.float64).sum(2) - 1)) < 1e-5


@settings(max_examples=40, deadline=None)
@given(arrays(np.float32, (8, 4, 4), elements=st.floats(-4, 4, width=32)),
       arrays(np.float32, (8, 4, 1), elements=st.floats(-4, 4, width=32)),
       arrays(np.float32, (8, 1, 4), elements=st.floats(-4, 4, width=32)))
def test_shift_invariance(R, a, b):
    T1 = oracle.birkhoff_proj_n4(R, 1e-7, threads=1)
    T2 = oracle.birkhoff_proj_n4((R + a + b).astype(np.float32), 1e-7, threads=1)
    assert np.max(np.abs(T1 - T2)) < 5e-5


@settings(max_examples=40, deadline=None)
@given(arrays(np.float32, (8, 4, 4), elements=st.floats(-3, 3, width=32)),
       arrays(np.float32, (8, 4, 4), elements=st.floats(-3, 3, width=32)))
def test_backward_rows_and_columns_sum_to_zero(R, G):
    T = oracle.birkhoff_proj_n4(R, 1e-7, threads=1)
    D = oracle.birkhoff_proj_n4_backward(G, T, threads=1)
    assert np.max(np.abs(D.astype(np.float64).sum(2))) < 1e-4
    assert np.max(np.abs(D.astype(np.float64).sum(1))) < 1e-4


@settings(max_examples=60, deadline=None)
@given(arrays(np.float32, (4, 4, 4), elements=any_float))
def test_any_input_terminates(R):
    T, ev = oracle.birkhoff_proj_n4(R, 1e-6, return_evals=True, threads=1)
    assert np.all(ev <= 3 + 20 * 7)
    assert T.shape == R.shape
