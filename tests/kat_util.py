"""Runs the reference-test known-answer cases (tests/golden/reference_kats.json)
against an implementation object exposing the reference kernel API in numpy
form (the oracle module, or the CUDA library's numpy front-end)."""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_cases():
    with open(os.path.join(HERE, "golden", "reference_kats.json")) as f:
        return json.load(f)["cases"]


def run_case(case, impl):
    op, x = case["op"], case["inputs"]
    arr = lambda k: np.asarray(x[k], np.float32)
    if op == "matmul":
        return impl.matmul(arr("A"), arr("B"), x["M"], x["N"], x["K"])
    if op == "relu_forward":
        return impl.relu_forward(arr("x"))
    if op == "relu_backward":
        return impl.relu_backward(arr("x"), arr("gy"))
    if op == "add":
        return impl.add(arr("a"), arr("b"))
    if op == "add_inplace":
        return impl.add_inplace(arr("a"), arr("b"))
    if op == "transpose":
        return impl.transpose(arr("x"), x["rows"], x["cols"])
    if op == "embedding_forward":
        ids = np.asarray(x["ids"], np.int32)
        return impl.embedding_forward(ids, arr("table"), arr("pos"), x["B"], x["S"], x["D"], x["V"], x["max_seq_len"])
    if op == "embedding_backward":
        ids = np.asarray(x["ids"], np.int32)
        return impl.embedding_backward(ids, arr("dout"), np.zeros(x["V"] * x["D"], np.float32),
                                       x["B"], x["S"], x["D"], x["V"])
    if op == "softmax":
        return impl.softmax(arr("x"), x["M"], x["N"])
    if op == "mha_causal_zeros":
        _, P = impl.mha_forward(arr("Q"), arr("K"), arr("V"), x["B"], x["S"], x["H"], x["Dh"], causal=True)
        S = x["S"]
        return np.array([P[i * S + j] for i, j in x["masked"]], np.float32)
    raise KeyError(op)


def check_case(case, impl):
    got = np.asarray(run_case(case, impl), np.float32)
    exp = np.asarray(case["expected"], np.float32)
    assert got.shape == exp.shape, (case["name"], got.shape, exp.shape)
    err = float(np.max(np.abs(got - exp))) if exp.size else 0.0
    assert err <= case["tol"], f"{case['name']} ({case['src']}): max abs err {err} > {case['tol']}"
