"""CPU tests: the line-tensor oracle against the server's own unit tests
(server/src/lines.rs:271-289), which fix the bucket geometry, the RGB
normalization and the zero right padding."""

import numpy as np
import pytest

from oracle import lines as OL


def test_line_geometry_golden():
    # lines.rs:271-278: bucket choice from the normalized width
    buckets = [128, 640, 960, 1280, 1600, 2400, 3200]

    def bucket_for(w, h):
        nat = OL.natural_width(w, h)
        fit = [b for b in buckets if b >= nat]
        if not fit:
            raise ValueError("exceeds")
        return fit[0]

    assert bucket_for(129, 48) == 640
    assert bucket_for(6400, 96) == 3200
    assert bucket_for(1, 48) == 128
    with pytest.raises(ValueError):
        bucket_for(3201, 48)
    with pytest.raises(ValueError):
        OL.natural_width(1, 0)


def test_line_tensor_preserves_rgb_and_padding_golden():
    # lines.rs:280-289
    image = np.zeros((48, 129, 3), np.uint8)
    image[...] = [0, 127, 255]
    t = OL.line_tensor(image, 640).reshape(-1)
    assert t[0] == -1.0
    assert t[2 * 48 * 640] == 1.0
    assert t[128] == -1.0
    assert t[129] == 0.0
    with pytest.raises(ValueError):
        OL.line_tensor(image, 128)
