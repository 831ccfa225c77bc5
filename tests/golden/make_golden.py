"""Generate the golden .weights fixtures with the reference's own quantizer.

Run in a container where the reference tree is mounted (it reads the reference's
python/src/tensor_io.py, save_tensor_with_header, python/src/tensor_io.py:40-321):

    python tests/golden/make_golden.py /path/to/cactus-reference

The fixtures are small (a few KB each) and committed; the tests only read them,
so the GPU box never needs the reference tree. Inputs are seeded float32 arrays
(numpy default_rng) plus hand-built edge cases: an all-zero group (scale floor
1e-10), and groups whose absmax is exactly 127 (INT8) or 7 (INT4) so that
w / scale lands on .5 ties and exercises round-half-to-even.
"""
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def cases():
    rng = np.random.default_rng(0)
    out = {}
    out["randn_16x256"] = (rng.standard_normal((16, 256), dtype=np.float32) * np.float32(0.02))
    out["randn_8x1024"] = (rng.standard_normal((8, 1024), dtype=np.float32) * np.float32(0.02))
    w = rng.standard_normal((4, 256), dtype=np.float32)
    w[1, :128] = 0.0  # all-zero groups at G=32 and G=128
    # exact ties: absmax 127 -> scale exactly 1.0; .5 values round half to even
    w[2, :] = np.float32(0.0)
    w[2, 0:8] = np.array([127.0, 2.5, -3.5, 0.5, -0.5, 1.5, -2.5, 126.5], np.float32)
    w[2, 32:40] = np.array([127.0, 4.5, -5.5, 6.5, 0.5, -1.5, 3.5, -126.5], np.float32)
    w[2, 128:136] = np.array([127.0, 2.5, -3.5, 0.5, -0.5, 1.5, -2.5, 126.5], np.float32)
    out["edge_4x256"] = w
    w4 = np.zeros((2, 64), np.float32)
    w4[0, 0:8] = np.array([7.0, 2.5, -3.5, 0.5, -0.5, 1.5, -2.5, 6.5], np.float32)  # scale exactly 1.0
    w4[1, :] = rng.standard_normal(64, dtype=np.float32)
    out["edge4_2x64"] = w4
    return out


def main(ref_root):
    sys.path.insert(0, str(Path(ref_root) / "python"))
    import src.tensor_io as tio  # reference quantizer

    manifest = {}
    for name, arr in cases().items():
        np.save(HERE / f"{name}.input.npy", arr)
        for prec in ("INT8", "INT4", "FP16"):
            for G in (32, 128):
                if prec == "FP16" and G == 128:
                    continue
                if arr.shape[1] % G:
                    continue
                tio.GROUP_SIZE = G
                fname = f"{name}.{prec.lower()}.g{G}.weights" if prec != "FP16" else f"{name}.fp16.weights"
                tio.save_tensor_with_header(arr, HERE / fname, precision=prec)
                manifest[fname] = {"input": f"{name}.input.npy", "precision": prec,
                                   "group_size": G if prec != "FP16" else 0}
    with open(HERE / "manifest.json", "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print(f"wrote {len(manifest)} fixtures to {HERE}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CACTUS_REFERENCE", ""))
