"""Writes tests/golden/known_answers.json.

The vectors restate the reference's own known-answer tests as data, by line of
jrm-code-project/llambda tests.lisp:

  T2386-2416  dequantize-q4-k-m: d=dmin=1.0, scales 2, mins 1, nibbles 6/7
              -> 11.0 for the low-nibble sub-blocks, 13.0 for the high ones
  T2418-2450  dequantize-q6-k: ql 0x31/0x42, qh 0xAA, scales 2, d=1.0
              -> 2, 4, 6, 8 per 32-value quarter of each 128-value chunk
  T2324-2367  the same blocks through load-gguf-tensor (11/13 and 2/8)
  T2257-2288  fused Q4_K row dot == dot of the dequantized row, x=((i mod 11)-5)/3
  T2290-2322  fused Q6_K row dot == dot of the dequantized row, x=((i mod 13)-6)/4
  T298-344    silu(2) = 1.7615942 (tolerance 1e-5); rms-norm values
  L4870-4874  the projection benchmark input x[i] = ((17 i + 11) mod 257)/128 - 1

Run:  python tests/golden/make_golden.py
"""
import json
import os


def q4k_block():
    b = [0] * 144
    b[0], b[1], b[2], b[3] = 0x00, 0x3C, 0x00, 0x3C  # d = dmin = 1.0 (fp16 LE)
    for i in range(4):
        b[4 + i] = 2        # scales 0..3 = 2
        b[8 + i] = 1        # mins 0..3 = 1
        b[12 + i] = 0x12    # scales 4..7 = 2 (low nibble), mins 4..7 = 1 (high)
    for i in range(128):
        b[16 + i] = 0x76    # low nibble 6, high nibble 7
    return b


def q6k_block():
    b = [0] * 210
    for i in range(32):
        b[i] = 0x31
        b[32 + i] = 0x42
        b[64 + i] = 0x31
        b[96 + i] = 0x42
    for i in range(64):
        b[128 + i] = 0xAA
    for i in range(16):
        b[192 + i] = 2
    b[208], b[209] = 0x00, 0x3C  # d = 1.0
    return b


def main():
    q4 = q4k_block()
    q6 = q6k_block()
    q4_expect = ([11.0] * 32 + [13.0] * 32) * 4
    q6_expect = ([2.0] * 32 + [4.0] * 32 + [6.0] * 32 + [8.0] * 32) * 2
    data = {
        "source": "jrm-code-project/llambda tests.lisp known-answer tests",
        "q4k_block": q4,
        "q4k_dequant": q4_expect,
        "q4k_dequant_checks": {"T2386-2416": {"0:32": 11.0, "32:64": 13.0,
                                              "192:224": 11.0, "224:256": 13.0},
                               "T2324-2367": {"0": 11.0, "32": 13.0}},
        "q6k_block": q6,
        "q6k_dequant": q6_expect,
        "q6k_dequant_checks": {"T2418-2450": {"0:32": 2.0, "32:64": 4.0, "64:96": 6.0,
                                              "96:128": 8.0, "128:160": 2.0,
                                              "224:256": 8.0},
                               "T2324-2367": {"0": 2.0, "96": 8.0}},
        "q4k_dot_x": [((i % 11) - 5) / 3.0 for i in range(256)],
        "q6k_dot_x": [((i % 13) - 6) / 4.0 for i in range(256)],
        "dot_tolerance": 1e-4,
        "silu_2": 1.7615942,
        "silu_tolerance": 1e-5,
        "rms_norm": {"x": [3.0, 4.0], "w": [1.0, 2.0], "eps": 0.0,
                     "expect": [0.84852815, 2.2627418]},
        "benchmark_input_rule": "x[i] = ((17*i + 11) mod 257)/128 - 1",
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(path, "w") as f:
        json.dump(data, f, indent=0)
    print("wrote", path)


if __name__ == "__main__":
    main()
