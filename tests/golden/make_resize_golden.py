"""Golden vectors for the image resize (OpenCV INTER_LINEAR, the cv2.resize
call of ResizeImages, fluxvla/transforms/transform_images.py:103-106).

    python tests/golden/make_resize_golden.py

Inputs are regenerated from their seeds by the tests; only the cv2 outputs
are stored (tests/golden/resize_u8.pt)."""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# (seed, src_h, src_w, dst_h, dst_w): the production 256 -> 224 downscale,
# an exact 2x downscale, an upscale, non-square and odd sizes
CASES = [(0, 256, 256, 224, 224), (1, 96, 96, 48, 48), (2, 20, 30, 28, 28),
         (3, 61, 47, 28, 42), (4, 128, 200, 112, 112)]


def source(seed, h, w):
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


def main():
    import cv2
    out = {}
    for seed, h, w, H, W in CASES:
        out[(seed, h, w, H, W)] = torch.from_numpy(
            cv2.resize(source(seed, h, w), (W, H), interpolation=cv2.INTER_LINEAR))
    torch.save({'cases': CASES, 'outputs': out, 'cv2': cv2.__version__},
               os.path.join(HERE, 'resize_u8.pt'))


if __name__ == '__main__':
    main()
