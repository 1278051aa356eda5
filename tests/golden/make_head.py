"""Calibrates the synthetic CTC head of the benchmark recognizer and writes
ppocrv6-native-server_b200/models/specs/recognizer_head.json.

The recognizer's weights are random (no PP-OCRv6 checkpoint is available
offline) and its inputs are U(-1,1) noise lines, as BASELINE config 4 asks.
Its hidden states are then dominated by one vector shared by every frame of
every line (the ReLU backbone's mean response carried through the 2048->120
projection and the residual stream), so a random vocabulary projection
decodes every frame to the same class. The head written here removes that
shared direction from the random projection and scales it so that the
frame-to-frame differences decide the argmax:

  W = gain * (I - u u^T) W0,    b = b0 + blank_bias * e_blank

with W0, b0 the seeded Xavier / normal draws (ppocr_b200.models.head_weights),
u the unit mean hidden vector of a seeded calibration batch (8 lines, run
through the CPU oracle of the same graph), gain chosen for a logit standard
deviation of 3 over the calibration frames and blank_bias for ~30 % blank
frames. The decoded lines then hold many distinct tokens, blanks and
repeats, which makes token-level parity a real test.

  python tests/golden/make_head.py
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "ppocrv6-native-server_b200"))
sys.path.insert(0, str(REPO))

LOGIT_STD = 3.0
BLANK_SHARE = 0.3


def main() -> None:
    import torch

    from ppocr_b200 import modelgen, models
    from oracle import models as OM

    spec = models.spec("recognizer")
    g, out = modelgen.build_recognizer(spec, 8, models.SEED)
    x = np.random.default_rng(models.SEED + 3).uniform(-1, 1, (8, 3, spec["height"], spec["width"]))
    hid, _ = OM.run_graph(g, x.astype(np.float32), out)
    h = hid.reshape(-1, hid.shape[-1]).double().numpy()
    center = h.mean(axis=0)
    u = center / np.linalg.norm(center)
    w0, b0 = models.head_weights(spec["neck"]["dim"], spec["vocab"], calibrated=False)
    wc = w0.astype(np.float64) - np.outer(u, u @ w0.astype(np.float64))
    logits = h @ wc
    gain = LOGIT_STD / logits.std()
    logits = gain * logits + b0
    blank = spec["blank"]
    others = np.delete(logits, blank, axis=1).max(axis=1)
    blank_bias = float(np.quantile(others - logits[:, blank], BLANK_SHARE))
    head = {
        "comment": "Synthetic CTC head calibration written by tests/golden/make_head.py: "
                   "W = gain * (I - u u^T) W0, b = b0 + blank_bias * e_blank, u = center / |center|.",
        "calibration": f"8 seeded U(-1,1) lines (seed {models.SEED + 3}) through the CPU oracle of the "
                       f"recognizer graph; logit std {LOGIT_STD}, blank share {BLANK_SHARE}",
        "gain": float(gain),
        "blank_bias": blank_bias,
        "center": [float(v) for v in center],
    }
    path = models.SPEC_DIR / "recognizer_head.json"
    path.write_text(json.dumps(head, indent=1) + "\n")
    w, b = models.head_weights(spec["neck"]["dim"], spec["vocab"])
    lg = h @ w.astype(np.float64) + b
    ids = lg.argmax(axis=1).reshape(8, -1)
    top2 = np.sort(lg, axis=1)[:, -2:]
    print(f"wrote {path}: gain {gain:.3f}, blank bias {blank_bias:.3f}; calibration frames: "
          f"{len(np.unique(ids))} distinct ids, blank share {(ids == blank).mean():.2f}, "
          f"top-2 gap > 1e-3 on {(top2[:, 1] - top2[:, 0] > 1e-3).mean():.3f} of frames")
    del torch


if __name__ == "__main__":
    main()
