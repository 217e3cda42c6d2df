"""Router outputs on which the reference's routing order and ranking by logit disagree.

k_route (engine/faie2fn.cu:1742-1800) ranks by v = expf(l - max l) in float32, equal v to the lower expert index.
Distinct logits can share one v; each case below builds such a tie in a way that does not depend on how the
exponential rounds (equal arguments, underflow to 0, saturation at 1), puts the smaller logit at the lower index, and
states the top-10 selection by hand.
"""

import numpy as np

F = np.float32


def collision_cases(ne=512):
    """[(logits float32 [ne], expected sel [10])]."""
    rng = np.random.default_rng(7)
    cases = []
    # equal arguments: l - 16 rounds to -15.5 for 0.5 and the floats just above it (spacing 2**-20 at 15.5)
    l = np.full(ne, -20.0, F)
    l[100] = 16.0
    for j, idx in enumerate([3, 7, 40, 41]):  # rising logits at rising indices: the logit order is 41, 40, 7, 3
        l[idx] = F(0.5) + F(j) * F(2.0 ** -24)
    cases.append((l, [100, 3, 7, 40, 41, 0, 1, 2, 4, 5]))
    # underflow: every v but the largest logit's is exactly 0, so the rest go by index
    l = rng.uniform(-10, 10, ne).astype(F)
    l[9] = 200.0
    cases.append((l, [9, 0, 1, 2, 3, 4, 5, 6, 7, 8]))
    # saturation at 1: l - m above -2**-25 gives v == 1
    l = np.full(ne, -5.0, F)
    top = F(2.0 ** -20)
    l[20] = top
    l[4] = top - F(2.0 ** -30)
    l[11] = top - F(2.0 ** -29)
    cases.append((l, [4, 11, 20, 0, 1, 2, 3, 5, 6, 7]))
    # two groups of equal arguments below a max of 8 (spacing 2**-21 at 7 and 7.5), larger logits at higher indices
    l = np.full(ne, -20.0, F)
    l[500] = 8.0
    l[2], l[10] = F(1.0), F(1.0) + F(2.0 ** -23)
    l[5], l[6] = F(0.5), F(0.5) + F(2.0 ** -24)
    cases.append((l, [500, 2, 10, 5, 6, 0, 1, 3, 4, 7]))
    return cases
