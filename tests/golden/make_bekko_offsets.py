"""Writes bekko_offsets.jsonl: token ids and byte offsets of texts, taken
from the reference's tokenizer fixture (testdata/bekko/offset_cases.jsonl of
github.com/bornholm/indecis, the outputs of its bekko tokenizer), with the
template's special tokens (first [2], last [1]) split off into "prefix" and
"suffix". The Spans tests use them as real tokenizations: token cores with
leading spaces, multi-byte runes, punctuation glued to words.

Usage: python tests/golden/make_bekko_offsets.py <reference checkout>
"""
import json
import os
import random
import sys


def main(ref: str):
    src = os.path.join(ref, "testdata", "bekko", "offset_cases.jsonl")
    rows = [json.loads(line) for line in open(src, encoding="utf-8")]
    for r in rows:
        assert r["ids"][0] == 2 and r["ids"][-1] == 1 and r["offsets"][0] == [0, 0] and r["offsets"][-1] == [0, 0]
    # Texts of 1 to 120 tokens, a fixed sample, plus the empty text.
    pool = [r for r in rows if 3 <= len(r["ids"]) <= 122]
    random.Random(20260101).shuffle(pool)
    pick = [r for r in rows if r["text"] == ""][:1] + pool[:160]
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "bekko_offsets.jsonl")
    with open(out, "w", encoding="utf-8") as f:
        for r in pick:
            f.write(json.dumps({"text": r["text"], "prefix": r["ids"][:1], "suffix": r["ids"][-1:],
                                "ids": r["ids"][1:-1], "offsets": r["offsets"][1:-1]}, ensure_ascii=False) + "\n")
    print(f"{len(pick)} texts -> {out}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("INDECIS_REFERENCE", "."))
