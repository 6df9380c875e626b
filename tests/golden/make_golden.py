"""Regenerate tinyblock_golden.json.

The fixtures are produced by a literal scalar restatement of the reference's
CPU QMV (nnmetal/src/transformer_test.zig:286-321) over weight buffers built
exactly like its createTestPackedBuffer helper (transformer_test.zig:886-923),
at TinyBlock shapes (transformer_test.zig:53-65).  They pin the vectorised
oracle in oracle/qwen3_ref.py.  Run: python tests/golden/make_golden.py
"""
import json
from pathlib import Path

import numpy as np


def packed_buffer(num_weights, seed):
    packed = np.array([(seed + i % 37) % 256 for i in range(num_weights // 8)], dtype=np.uint8)
    scales = np.array([0.1 + (seed % 10) * 0.01 + i * 0.005 for i in range(num_weights // 128)],
                      dtype=np.float32).astype(np.float16)
    return packed, scales


def cpu_qmv(bits, scales, x, M, K, gs=128):
    out = []
    for row in range(M):
        acc = np.float32(0.0)
        for col in range(K):
            flat = row * K + col
            bit = (int(bits[flat // 8]) >> (flat % 8)) & 1
            s = np.float32(scales[flat // gs])
            acc = np.float32(acc + np.float32((s if bit else -s) * np.float32(x[col])))
        out.append(float(acc))
    return out


def main():
    cases = []
    for (M, K, seed) in [(128, 128, 1), (256, 128, 2), (128, 256, 5)]:  # q/k/v, gate, down
        bits, scales = packed_buffer(M * K, seed)
        x = [float(np.float32(np.sin(0.1 * i + seed))) for i in range(K)]
        cases.append({"M": M, "K": K, "seed": seed, "x": x, "y": cpu_qmv(bits, scales, x, M, K)})
    out = Path(__file__).with_name("tinyblock_golden.json")
    out.write_text(json.dumps({"source": "literal cpuQMV over createTestPackedBuffer", "qmv": cases}))
    print(out)


if __name__ == "__main__":
    main()
