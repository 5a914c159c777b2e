"""Known-answer tests of the routing rule (reference/moe_ref.py:82-107) on the CPU oracle.

Exact ties follow the lower-index convention of the reference CUDA kernel
(kernels/moe.cu:146-158 warp argmax, :261-273 group pick, :276-305 expert pick).
The same cases run against the device router in tests/test_gpu_route.py.
"""
import numpy as np
import pytest

T_KAT = 6


def kat_cases():
    """(name, logits [T,256], bias [256], expected sorted top-8 per token)."""
    cases = []
    # 1. all-equal logits, zero bias: every score ties -> groups 0-3, experts 0..7.
    lg = np.zeros((1, 256), np.float32)
    cases.append(("all_equal", lg, np.zeros(256, np.float32), [list(range(8))]))
    # 2. a clear winner per group order: group g gets logit 2-g/10 on its first 8 experts.
    lg = np.full((1, 256), -4.0, np.float32)
    for g in range(8):
        lg[0, 32 * g:32 * g + 8] = 2.0 - g / 10.0
    cases.append(("group_order", lg, np.zeros(256, np.float32), [list(range(8))]))
    # 3. hot bias on experts {32g, 32g+1}: the biased top-2 of every group are the hot pair;
    #    groups 0-3 win the tie on group score -> experts 0,1,32,33,64,65,96,97.
    b = np.zeros(256, np.float32)
    for g in range(8):
        b[32 * g] = b[32 * g + 1] = 1.5
    cases.append(("hot_bias", np.zeros((1, 256), np.float32), b, [[0, 1, 32, 33, 64, 65, 96, 97]]))
    # 4. group pruning: the 9 best single scores sit in one group, but that group's top-2 sum
    #    is lower than four others' -> those experts are excluded.
    lg = np.full((1, 256), -6.0, np.float32)
    lg[0, 224:256] = -6.0
    lg[0, 224] = 3.0                       # group 7: top-2 = 3.0 + (-6) -> low group score
    for g in range(4):
        lg[0, 32 * g:32 * g + 2] = 1.0     # groups 0-3: top-2 sum = 2 * sigmoid(1)
    cases.append(("group_pruning", lg, np.zeros(256, np.float32), [[0, 1, 32, 33, 64, 65, 96, 97]]))
    # 5. tie at the 8th place inside kept groups -> lower index wins.
    #    Seven scores above the tied pair: 0..4 (group 0), 33 (group 1), 64 (group 2); group 3
    #    ties groups 4-7 on score and is kept as the lowest of them.
    lg = np.full((1, 256), -5.0, np.float32)
    lg[0, [0, 1, 2, 3, 4]] = 3.0
    lg[0, [33, 64]] = 2.5
    lg[0, [40, 8]] = 1.0                    # 8 and 40 tie for the last slot; 8 is lower
    cases.append(("tie_8th", lg, np.zeros(256, np.float32), [[0, 1, 2, 3, 4, 8, 33, 64]]))
    return cases


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c[0])
def test_route_kat(case, oracle):
    name, lg, b, expect = case
    idx, w = oracle.route(lg, b, 2.5)
    if expect is not None:
        assert np.sort(idx, axis=1).tolist() == expect
    # selection order: non-increasing biased score
    s = oracle.sigmoid_rn(lg) + b
    sel = np.take_along_axis(s, idx, axis=1)
    assert (np.diff(sel, axis=1) <= 0).all()
    np.testing.assert_allclose(w.sum(axis=1), 2.5, rtol=1e-5)


def test_tie_8th_lower_index(oracle):
    case = [c for c in kat_cases() if c[0] == "tie_8th"][0]
    idx, _ = oracle.route(case[1], case[2], 1.0)
    chosen = set(idx[0].tolist())
    assert 8 in chosen and 40 not in chosen


def test_weights_use_unbiased_scores(oracle):
    """w = sigmoid(logit) / sum over the 8 picks * rsf, with the bias only used to select."""
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((32, 256)).astype(np.float32)
    b = (0.3 * rng.standard_normal(256)).astype(np.float32)
    idx, w = oracle.route(lg, b, 2.5)
    s = oracle.sigmoid_rn(lg)
    ss = np.take_along_axis(s, idx, axis=1)
    np.testing.assert_allclose(w, ss / ss.sum(axis=1, keepdims=True) * 2.5, rtol=1e-6)
