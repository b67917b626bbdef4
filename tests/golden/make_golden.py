"""Generate tests/golden/golden.json: SHA-256 digests of oracle outputs on small
seeded cases (run: ``python -m tests.golden.make_golden``).

The digests pin the oracle's bits across machines (glibc libm version, compiler
flags): the oracle test recomputes every case and requires the same digest,
and the GPU parity tests compare the CUDA outputs against the same digests.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

from tests import _data

HERE = os.path.dirname(os.path.abspath(__file__))


def _h(*arrays) -> str:
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()


def inputs():
    """The seeded inputs behind every golden case (shared with the GPU tests)."""
    d = {}
    d["rms_x"] = _data.lcg_normal(7 * 576, 21).reshape(7, 576)
    d["rms_w"] = _data.lcg_normal(576, 22, 1.0, 0.1)
    d["qk_v"] = _data.lcg_normal(5 * 1024, 23).reshape(5, 1024)
    d["qk_w"] = _data.lcg_normal(128, 24, 1.0, 0.1)
    d["rope_q"] = _data.lcg_normal(6 * 576, 25).reshape(6, 576)
    d["rope_k"] = _data.lcg_normal(6 * 192, 26).reshape(6, 192)
    d["rope_pos"] = np.array([0, 1, 2, 127, 511, 4095], np.uint64)
    d["silu_g"] = _data.lcg_normal(3000, 27, 0.0, 4.0)
    d["silu_u"] = _data.lcg_normal(3000, 28)
    d["conv_x"] = _data.lcg_normal(9 * 40, 29).reshape(9, 40)
    d["conv_w"] = _data.lcg_normal(40 * 3, 30, 0.0, 0.3)
    d["q8_x"] = _data.lcg_normal(3 * 1000, 31).reshape(3, 1000)
    d["emb_bf16"] = _data.bf16_table(64, 96, 32)
    d["emb_q8"], d["emb_q8_s"] = _data.q8_table(64, 96, 33)
    d["emb_tok"] = _data.tokens(17, 64, 34)
    return d


def compute(oracle) -> dict:
    d = inputs()
    c = {}
    c["rms_norm_576"] = _h(oracle.rms_norm(d["rms_x"], d["rms_w"], 1e-5))
    c["qk_norm_128"] = _h(oracle.qk_norm(d["qk_v"], 128, d["qk_w"], 1e-6))
    q, k = oracle.rope(d["rope_q"], d["rope_k"], d["rope_pos"], 64, 1e5, interleaved=False)
    c["rope_half_64"] = _h(q, k)
    q, k = oracle.rope(d["rope_q"], d["rope_k"], d["rope_pos"], 64, 1e5, interleaved=True)
    c["rope_pair_64"] = _h(q, k)
    c["silu_mul"] = _h(oracle.silu_mul(d["silu_g"], d["silu_u"]))
    c["conv_prefill_k3"] = _h(oracle.conv_prefill(d["conv_x"], d["conv_w"], 3))
    c["q8_quantize"] = _h(*oracle.q8_quantize_rows(d["q8_x"]))
    c["embed_bf16"] = _h(oracle.embed_rows(oracle.BF16, d["emb_bf16"], None, 64, 96, d["emb_tok"]))
    c["embed_q8_0"] = _h(
        oracle.embed_rows(oracle.Q8_0, d["emb_q8"], d["emb_q8_s"], 64, 96, d["emb_tok"]))
    return c


def main():
    from oracle import oracle

    out = {"generator": "tests/golden/make_golden.py", "cases": compute(oracle)}
    with open(os.path.join(HERE, "golden.json"), "w") as fh:
        json.dump(out, fh, indent=1, sort_keys=True)
        fh.write("\n")


if __name__ == "__main__":
    main()
