"""CPU check of the CSV decoder's feature rule (dp_csv_parse_feature: the
host build of the code every GPU cell runs, csrc/dec2f.cuh) against the
reference's own feature() (native/decision_programs_csv.hpp:28-34, run by
oracle/_ref/ref_csv --tokens): acceptance and binary32 bits for random
decimals, exact binary32 midpoints written out in full and perturbed in their
last digit, range boundaries and malformed tokens."""
import ctypes
import pathlib
import random
import struct
import subprocess
from decimal import Decimal, getcontext
from fractions import Fraction

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref" / "ref_csv"

pytestmark = pytest.mark.skipif(not REF.exists(), reason="reference CSV harness not built (needs the reference sources)")

SPECIAL = ["", " ", "nan", "NaN", "NA", "na", "null", "NULL", "Null", "inf", "-inf", "infinity", "-nan", "1e", "1e+",
           "+", "-", "+-5", "-+5", ".", ".5", "5.", "e5", "0x1", "1_0", " 7 ", "\t-3.5\r", "++1", "1.5.2", "--1",
           "0e999999", "1e-999999", "00000.000", "-0", "-0.0e10", "1E5", "1e+05", "3.4028235e38", "3.4028236e38",
           "1e-45", "7e-46", "1.4e-45", "0.000001e-39", "123456789012345678901234567890", "1" + "0" * 300,
           "0." + "0" * 300 + "1", "1,5", "1 5", '"1"', "\v1\f", "١"]


def float_bits(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", f))[0]


def exact_decimal(fr: Fraction, digits: int) -> str:
    getcontext().prec = digits
    return format(Decimal(fr.numerator) / Decimal(fr.denominator), "e")


def tokens(n: int, seed: int) -> list[str]:
    rng = random.Random(seed)
    out = list(SPECIAL)
    for _ in range(n):
        k = rng.randrange(6)
        if k == 0:  # exact midpoint between a binary32 and its successor
            b = rng.randrange(0x7f7fffff)
            lo = Fraction(struct.unpack("<f", struct.pack("<I", b))[0])
            hi = Fraction(struct.unpack("<f", struct.pack("<I", b + 1))[0])
            s = exact_decimal((lo + hi) / 2, 140)
            mant, exp = s.split("e")
            cut = rng.randrange(len(mant) + 1)
            variants = [s, mant[:max(cut, 3)] + "e" + exp]
            t = mant[:max(cut, 3)]
            if t[-1].isdigit() and t[-1] != "9":
                variants.append(t[:-1] + chr(ord(t[-1]) + 1) + "e" + exp)
            out += variants
        elif k == 1:
            b = rng.randrange(0x7f800000)
            out.append(f"{struct.unpack('<f', struct.pack('<I', b))[0]:.{rng.randrange(3, 12)}e}")
        elif k == 2:
            out.append(str(rng.randrange(10**rng.randrange(1, 30))) + "." + str(rng.randrange(10**rng.randrange(1, 12))))
        elif k == 3:
            out.append(f"{rng.uniform(-1e6, 1e6):.{rng.randrange(0, 12)}f}")
        elif k == 4:
            out.append(f"{rng.randrange(1, 10**7)}e{rng.randrange(-60, 45)}")
        else:
            out.append(rng.choice(["-", "+", " ", ""]) + str(rng.random()) + rng.choice(["", "e3", "e-50", "x"]))
    return out


def test_feature_tokens_match_reference(dp, tmp_path):
    toks = tokens(40_000, 11)
    toks = [t for t in toks if "\n" not in t]
    src = tmp_path / "tokens.txt"
    src.write_bytes(b"".join(t.encode() + b"\n" for t in toks))
    out = tmp_path / "ref.txt"
    subprocess.run([str(REF), "--tokens", str(src), str(out)], check=True, timeout=300)
    ref = out.read_text().splitlines()
    assert len(ref) == len(toks)
    lib = dp.lib()
    v = ctypes.c_float()
    accepted = 0
    for t, r in zip(toks, ref):
        b = t.encode()
        rc = lib.dp_csv_parse_feature(b, len(b), ctypes.byref(v))
        if r == "0":
            assert rc == 1, (t, float_bits(v.value))
        else:
            accepted += 1
            assert rc == 0, t
            assert f"{float_bits(v.value):08x}" == r.split()[1], (t, f"{float_bits(v.value):08x}", r)
    assert accepted > len(toks) // 2
