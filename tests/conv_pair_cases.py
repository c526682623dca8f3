"""Stride-1 convolutions that the CTA-pair halo forward serves (enough pair tiles for the
GPU's TPCs): config 4's forward and input gradient in TF32 and 3xTF32, and a shape whose
row of tiles is odd, so the last pair's second tile lies past the right edge. Run directly,
it writes each output and its path to the .npz named on the command line; MT_CONV_PAIR is
read once per process, so each setting needs its own process."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from minitensor_b200 import engine, inputs  # noqa: E402


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_cases():
    out, paths = {}, {}
    x, w, b, dy = inputs.config4()
    xd, wd, bd, dyd = _dev(x), _dev(w), _dev(b), _dev(dy)
    # 16 x 64 x 40 x 42: 8 x 14 tiles -> 3 per row (odd), 5 rows, 16 images = 160 pair tiles.
    x2 = _dev(inputs.normal((16, 64, 40, 42), 1.0, 1801))
    w2 = _dev(inputs.normal((64, 64, 3, 3), 0.06, 1802))
    b2 = _dev(inputs.normal((64,), 0.1, 1803))
    for mode in ("tf32", "tf32x3"):
        y = engine.conv2d(xd, wd, bd, 1, 1, mode=mode)
        out[f"fwd_{mode}"], paths[f"fwd_{mode}"] = y.cpu().numpy(), engine.last_path()
        dx, _, _ = engine.conv2d_backward(dyd, xd, wd, 1, 1, need=("input",), mode=mode)
        out[f"dgrad_{mode}"], paths[f"dgrad_{mode}"] = dx.cpu().numpy(), engine.last_path()
        y2 = engine.conv2d(x2, w2, b2, 1, 1, mode=mode)
        out[f"odd_{mode}"], paths[f"odd_{mode}"] = y2.cpu().numpy(), engine.last_path()
    torch.cuda.synchronize()
    return out, paths


if __name__ == "__main__":
    torch.cuda.set_device(0)
    engine.lib()
    o, p = run_cases()
    np.savez(sys.argv[1], **o, **{"path_" + k: np.array(v) for k, v in p.items()})
