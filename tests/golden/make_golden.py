"""Writes tests/golden/reference_kats.json: the known-answer cases of the
reference's own kernel tests (buladuo/ZeroLLM tests/kernel_*.cpp).

Each case restates the test's input construction and records the expected
output the test states (hand values) or derives by hand-evaluable rules
(embedding/transpose).  Cases cite file:line in the reference project.
Run from the repository root:  python tests/golden/make_golden.py
"""
import json
import os

import numpy as np


def f32pos(i, j):
    """float(i + j * 0.1f) evaluated in float32 as in the C++ test."""
    return float(np.float32(i) + np.float32(j) * np.float32(0.1))

cases = []


def case(name, src, op, inputs, expected, tol):
    cases.append({"name": name, "src": src, "op": op, "inputs": inputs, "expected": expected, "tol": tol})


# kernel_matmul.cpp:55-83  A=[[1,2],[3,4],[5,6]] (3x2), B=[[1..4],[5..8]] (2x4)
case("matmul_kat", "tests/kernel_matmul.cpp:55-83", "matmul",
     {"A": [float(i + 1) for i in range(6)], "B": [float(i + 1) for i in range(8)], "M": 3, "N": 4, "K": 2},
     [11, 14, 17, 20, 23, 30, 37, 44, 35, 46, 57, 68], 1e-3)

# kernel_relu.cpp:20-30 positive values pass through
case("relu_fwd_positive", "tests/kernel_relu.cpp:20-30", "relu_forward",
     {"x": [float(i + 1) for i in range(10)]}, [float(i + 1) for i in range(10)], 1e-6)
# kernel_relu.cpp:80-81
case("relu_fwd_mixed", "tests/kernel_relu.cpp:80-81", "relu_forward",
     {"x": [-3.0, -1.0, 0.0, 1.0, 2.0, -0.5, 4.0, -2.0, 0.0, 5.0]},
     [0.0, 0.0, 0.0, 1.0, 2.0, 0.0, 4.0, 0.0, 0.0, 5.0], 1e-6)
# kernel_relu.cpp:199-202
case("relu_bwd_ones", "tests/kernel_relu.cpp:199-202", "relu_backward",
     {"x": [-1.0, 2.0, -3.0, 0.0, 4.0, -5.0], "gy": [1.0] * 6},
     [0.0, 1.0, 0.0, 0.0, 1.0, 0.0], 1e-6)
# kernel_relu.cpp:262-265
case("relu_bwd_values", "tests/kernel_relu.cpp:262-265", "relu_backward",
     {"x": [1.0, -2.0, 3.0, 0.0, -4.0, 5.0, -0.5, 0.0], "gy": [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8]},
     [0.1, 0.0, 0.3, 0.0, 0.0, 0.6, 0.0, 0.0], 1e-6)

# kernel_add.cpp:29-31, :206-208, :261-263
case("add_kat", "tests/kernel_add.cpp:29-31", "add",
     {"a": [float(i + 1) for i in range(10)], "b": [float(10 - i) for i in range(10)]}, [11.0] * 10, 1e-6)
case("add_negatives", "tests/kernel_add.cpp:206-208", "add",
     {"a": [-1.0, -2.0, -3.0, -4.0, -5.0], "b": [1.0, 2.0, 3.0, 4.0, 5.0]}, [0.0] * 5, 1e-6)
case("add_inplace_kat", "tests/kernel_add.cpp:261-263", "add_inplace",
     {"a": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], "b": [6.0, 5.0, 4.0, 3.0, 2.0, 1.0]}, [7.0] * 6, 1e-6)

# kernel_transpose.cpp:22-43 (3x4 of 1..12) and :95-109 (4x4 of 0..15)
case("transpose_3x4", "tests/kernel_transpose.cpp:22-43", "transpose",
     {"x": [float(i + 1) for i in range(12)], "rows": 3, "cols": 4},
     [1, 5, 9, 2, 6, 10, 3, 7, 11, 4, 8, 12], 1e-6)
case("transpose_4x4", "tests/kernel_transpose.cpp:95-109", "transpose",
     {"x": [float(i) for i in range(16)], "rows": 4, "cols": 4},
     [0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15], 1e-6)

# kernel_embedding.cpp:22-70: ids {1..6}, table[i,j]=i*D+j, pos[s,j]=s+0.1j, expected table[id]+pos[s]
B, S, D, V, MS = 2, 3, 4, 10, 5
table = [float(i * D + j) for i in range(V) for j in range(D)]
pos = [f32pos(i, j) for i in range(MS) for j in range(D)]
ids = [1, 2, 3, 4, 5, 6]
exp = []
for b in range(B):
    for s in range(S):
        for j in range(D):
            exp.append(float(np.float32(table[ids[b * S + s] * D + j]) + np.float32(pos[s * D + j])))
case("embedding_fwd", "tests/kernel_embedding.cpp:22-70", "embedding_forward",
     {"ids": ids, "table": table, "pos": pos, "B": B, "S": S, "D": D, "V": V, "max_seq_len": MS}, exp, 1e-6)

# kernel_embedding.cpp:123-170: ids {1,2,1,2,1,2}, dout[i] = i%5+1, dtable starts at 0
ids = [1, 2, 1, 2, 1, 2]
dout = [float(i % 5 + 1) for i in range(B * S * D)]
dt = [0.0] * (V * D)
for t in range(B * S):
    for j in range(D):
        dt[ids[t] * D + j] += dout[t * D + j]
case("embedding_bwd", "tests/kernel_embedding.cpp:123-170", "embedding_backward",
     {"ids": ids, "dout": dout, "B": B, "S": S, "D": D, "V": V}, dt, 1e-6)

# kernel_embedding.cpp:216-275: ids {-1,2,10}; rows of invalid ids stay 0
table = [float(i * 2 + j) for i in range(5) for j in range(2)]
pos = [f32pos(i, j) for i in range(3) for j in range(2)]
exp = [0.0, 0.0, float(np.float32(table[4]) + np.float32(pos[2])), float(np.float32(table[5]) + np.float32(pos[3])), 0.0, 0.0]
case("embedding_invalid_ids", "tests/kernel_embedding.cpp:216-275", "embedding_forward",
     {"ids": [-1, 2, 10], "table": table, "pos": pos, "B": 1, "S": 3, "D": 2, "V": 5, "max_seq_len": 3}, exp, 0.0)

# kernel_softmax.cpp:240-262: rows of 0, 100, -100 -> uniform
case("softmax_edge_rows", "tests/kernel_softmax.cpp:240-262", "softmax",
     {"x": [0.0] * 4 + [100.0] * 4 + [-100.0] * 4, "M": 3, "N": 4}, [0.25] * 12, 1e-5)

# kernel_mha.cpp:140-213: causal, B=1,S=3,H=1,Dh=2; probabilities (0,1),(0,2),(1,2) ~ 0
case("mha_causal_mask", "tests/kernel_mha.cpp:140-213", "mha_causal_zeros",
     {"Q": [1, 0, 0, 1, 1, 1], "K": [1, 0, 0, 1, 1, 1], "V": [1, 2, 3, 4, 5, 6], "B": 1, "S": 3, "H": 1, "Dh": 2,
      "masked": [[0, 1], [0, 2], [1, 2]]}, [0.0, 0.0, 0.0], 1e-4)

out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
with open(out, "w") as f:
    json.dump({"source": "buladuo/ZeroLLM tests/kernel_*.cpp", "cases": cases}, f, indent=1)
print(f"wrote {len(cases)} cases to {out}")
