"""oracle/decode.py pinned to the reference's own pose decoder and NMS.

tests/golden/decode_vectors.npz holds outputs of src/Decoders.cpp
(`PoseDecoder::decode`, `nmsPerClass`) and src/Nms.cpp, compiled from the
reference sources (generator: tests/golden/make_decode_golden.py; build
recipe: `make -C oracle ref`), on synthetic, adversarial and network outputs.
The restatement must give the same detections in the same order with the same
float values (score, box, keypoints).  The device decode (ivc_decode_pose) is
checked bit for bit against the restatement in tests/test_gpu_decode.py."""
import os

import numpy as np
import pytest

from oracle import decode

GOLD = os.path.join(os.path.dirname(__file__), "golden", "decode_vectors.npz")
_g = np.load(GOLD)
CASES = sorted({k.split("/")[0] for k in _g.files})


@pytest.mark.parametrize("name", CASES)
def test_decode_matches_reference(name):
    out = _g[f"{name}/out"].astype(np.float32)
    conf, iou, max_det, scale, pl, pt = _g[f"{name}/params"]
    ref = _g[f"{name}/dets"]
    got = decode.pose_decode(out, conf=float(np.float32(conf)), iou=float(np.float32(iou)), max_det=int(max_det),
                             nk=17, kdims=3, scale=float(np.float32(scale)), pad=(int(pl), int(pt)))
    assert len(got) == len(ref), (name, len(got), len(ref))
    for k, (a, score, box, kp) in enumerate(got):
        row = np.concatenate([[score], box, kp.reshape(-1)]).astype(np.float32)
        assert np.array_equal(row, ref[k]), (name, k, a, row[:5], ref[k][:5])
