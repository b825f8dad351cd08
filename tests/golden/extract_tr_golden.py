"""Extract TR's golden dequant vectors into tr_golden.json.

Reads sekerahmet/TCB's internal/compute/tensor/quant_test.go as text (the
table of TestDequantMatchesLlamaCpp, quant_test.go:55-87, whose hashes TR
took from llama.cpp's dequantize_row_* run on the same bytes) and writes
the entries next to this script.  Run where the reference checkout exists:

    python tests/golden/extract_tr_golden.py /path/to/TCB
"""
import json
import os
import re
import sys

NAMES = {"Q8": "q8_0", "Q4K": "q4_k", "Q6K": "q6_k", "Q4": "q4_0"}


def main(root: str) -> None:
    src = os.path.join(root, "internal/compute/tensor/quant_test.go")
    text = open(src, encoding="utf-8").read()
    body = text[text.index("func TestDequantMatchesLlamaCpp"):]
    body = body[: body.index("t.Run(")]
    rows = re.findall(r"\{(Q8|Q4K|Q6K|Q4), (\d+), (0x[0-9a-f]+), (\d+), (0x[0-9a-f]+)\}", body)
    if len(rows) != 4:
        raise SystemExit(f"expected 4 golden rows, found {len(rows)}")
    blocks = int(re.search(r"const quantTestBlocks = (\d+)", text).group(1))
    out = {
        "source": "internal/compute/tensor/quant_test.go:55-87 (TestDequantMatchesLlamaCpp)",
        "generator": "internal/compute/tensor/quant_test.go:20-45 (randomQuant LCG)",
        "blocks": blocks,
        "cases": [
            {"format": NAMES[dt], "seed": int(seed), "fnv1a64": hx, "at": int(at), "sample_bits": sm}
            for dt, seed, hx, at, sm in rows
        ],
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tr_golden.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: extract_tr_golden.py <TR source tree>")
    main(sys.argv[1])
