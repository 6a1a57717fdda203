"""oracle/preprocess.py pinned to the reference's image preprocessing.

tests/golden/preprocess_vectors.npz holds the output of src/Preprocess.cpp's
steps run with the OpenCV calls it makes (generator:
tests/golden/make_preprocess_golden.py); the restatement must reproduce every
blob value and the letterbox geometry exactly."""
import os

import numpy as np
import pytest

from oracle import preprocess

GOLD = os.path.join(os.path.dirname(__file__), "golden", "preprocess_vectors.npz")
_g = np.load(GOLD)
CASES = sorted({k.split("/")[0] for k in _g.files})


@pytest.mark.parametrize("name", CASES)
def test_preprocess_matches_reference(name):
    ih, iw, lb, rgb, norm = (int(v) for v in _g[f"{name}/params"])
    blob, info = preprocess.preprocess(_g[f"{name}/image"], ih, iw, letterbox=bool(lb), to_rgb=bool(rgb),
                                       normalize=bool(norm), mean=tuple(_g[f"{name}/mean"]),
                                       std=tuple(_g[f"{name}/std"]))
    assert np.array_equal(blob, _g[f"{name}/blob"]), name
    assert np.array_equal(np.array(info, np.float32), _g[f"{name}/letterbox"]), (info, _g[f"{name}/letterbox"])
