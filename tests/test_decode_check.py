"""The NMS-set check itself (CPU): `oracle.decode.undecided_anchors` must bound
every change of the post-NMS set that a bounded perturbation of the head output
can cause, and be empty when nothing is perturbed."""
import numpy as np
import pytest

from oracle import decode


def synthetic_head(rng, anchors=1500, clusters=300):
    """[56, A] head output with clustered boxes (IoUs around the 0.7 threshold)
    and scores spread across the 0.25 confidence threshold."""
    out = np.zeros((56, anchors), dtype=np.float32)
    centers = rng.uniform(50, 590, size=(clusters, 2))
    sizes = rng.uniform(20, 150, size=(clusters, 2))
    c = rng.integers(0, clusters, anchors)
    out[0] = centers[c, 0] + rng.normal(0, 8, anchors)
    out[1] = centers[c, 1] + rng.normal(0, 8, anchors)
    out[2] = sizes[c, 0] * rng.uniform(0.8, 1.2, anchors)
    out[3] = sizes[c, 1] * rng.uniform(0.8, 1.2, anchors)
    out[4] = rng.beta(0.5, 3.0, anchors)
    out[5:] = rng.uniform(0, 640, size=(51, anchors))
    return out.astype(np.float16).astype(np.float32)


def ids(out, **kw):
    return {a for a, *_ in decode.pose_decode(out, **kw)}


@pytest.mark.parametrize("seed", range(12))
def test_undecided_bounds_set_changes(seed):
    rng = np.random.default_rng(seed)
    ref = synthetic_head(rng)
    for scale_s, scale_b in [(1e-3, 0.05), (4e-3, 0.25), (2e-2, 1.0)]:
        cmp_ = ref.copy()
        cmp_[4] += rng.uniform(-scale_s, scale_s, ref.shape[1]).astype(np.float32)
        cmp_[:4] += rng.uniform(-scale_b, scale_b, (4, ref.shape[1])).astype(np.float32)
        for kw in ({}, {"max_det": 40}):
            und, delta, eps = decode.undecided_anchors(ref, cmp_, **kw)
            diff = ids(ref, **kw) ^ ids(cmp_, **kw)
            assert diff <= und, (sorted(diff - und)[:5], delta, eps)
            if scale_s == 1e-3 and not kw:  # the bound stays selective at small deviations
                assert len(und) < 0.25 * int((ref[4] >= 0.25).sum()), len(und)


def test_undecided_empty_without_perturbation():
    rng = np.random.default_rng(99)
    ref = synthetic_head(rng, anchors=600)
    # distinct scores (no greedy-order ties): distinct fp16 values in (0, 1)
    grid = np.arange(0x1400, 0x3C00, dtype=np.uint16).view(np.float16)
    ref[4] = rng.choice(grid, ref.shape[1], replace=False).astype(np.float32)
    und, delta, eps = decode.undecided_anchors(ref, ref.copy())
    assert delta == 0.0 and eps == 0.0
    assert und == set()
