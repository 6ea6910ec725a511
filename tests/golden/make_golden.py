"""Writes reference_known_answers.json: the reference's own CPU-checked
fixtures, restated from its JNI suite
(runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala):

  vectorAdd (:114-122):  left(i) = i.toFloat, right(i) = (i*2).toFloat,
                         n = 1024, expected(i) = left(i) + right(i), exact.
  blockReduceSum (:235-238, :310): input(i) = (i % 8).toFloat, n = 256,
                         expected = inputValues.sum (sequential Float fold).

Run: python tests/golden/make_golden.py
"""
import json
from pathlib import Path

import numpy as np


def main() -> None:
    n_add = 1024
    left = np.arange(n_add, dtype=np.float32)
    right = (np.arange(n_add) * 2).astype(np.float32)
    expected_add = (left + right).astype(np.float32)

    n_sum = 256
    values = (np.arange(n_sum) % 8).astype(np.float32)
    acc = np.float32(0.0)
    for v in values:  # Scala Array[Float].sum: left fold in Float
        acc = np.float32(acc + v)

    out = {
        "vector_add": {"n": n_add, "left": "i", "right": "2*i",
                       "expected_first": expected_add[:8].tolist(),
                       "expected_sum_of_outputs": float(expected_add.astype(np.float64).sum())},
        "block_reduce_sum": {"n": n_sum, "input": "i % 8", "expected": float(acc)},
    }
    path = Path(__file__).with_name("reference_known_answers.json")
    path.write_text(json.dumps(out, indent=2) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
