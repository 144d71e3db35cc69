"""The GPU CSV input transport (dp_csv_decode) against the reference's own
decision_programs_csv::decode (native/decision_programs_csv.hpp:36-67,
compiled unmodified into oracle/_ref/ref_csv): the same values bit for bit,
labels, class counts, header decisions, feature names and label mappings, and
the same error messages, on edge cases of the CSV grammar, of the feature
tokens and of class labels, and on seeded random tables."""
import json
import pathlib
import random
import struct
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref" / "ref_csv"
needs_ref = pytest.mark.skipif(not REF.exists(), reason="reference CSV harness not built (needs the reference sources)")


def reference(tmp_path, data: bytes, target: str, header: str):
    src = tmp_path / "in.csv"
    src.write_bytes(data)
    out = tmp_path / "ref"
    out.mkdir(exist_ok=True)
    for f in out.iterdir():
        f.unlink()
    subprocess.run([str(REF), str(src), target or "-", header, str(out)], check=True, timeout=120)
    if (out / "error.txt").exists():
        return {"error": (out / "error.txt").read_text()}
    meta = json.loads((out / "meta.json").read_text())
    meta["values"] = np.fromfile(out / "values.f32", dtype="<u4")
    meta["labels"] = np.fromfile(out / "labels.u32", dtype="<u4")
    return meta


def ours(dp, data: bytes, target: str, header: str):
    try:
        t = dp.CsvTable(data, target, header)
    except dp.DPError as e:
        return {"error": str(e)}
    v, lb = t.to_numpy()
    r = {"rows": t.rows, "features": t.features, "classes": t.classes, "header": t.header, "names": t.names,
         "label_mapping": t.label_mapping, "values": v.reshape(-1).view(np.uint32),
         "labels": lb if lb is not None else np.zeros(0, np.uint32)}
    t.free()
    return r


def same(dp, tmp_path, data: bytes, target: str = "", header: str = "auto"):
    want = reference(tmp_path, data, target, header)
    got = ours(dp, data, target, header)
    if "error" in want:
        assert "error" in got, (data[:200], want["error"])
        assert want["error"] in got["error"], (got["error"], want["error"])
        return want
    assert "error" not in got, (data[:200], got["error"])
    for k in ("rows", "features", "classes", "header", "names", "label_mapping"):
        assert got[k] == want[k], (k, got[k], want[k])
    np.testing.assert_array_equal(got["values"], want["values"])
    np.testing.assert_array_equal(got["labels"], want["labels"])
    return want


EDGE = [
    (b"a,b,y\n1.5,2,x\n3,4,y\n", "y", "auto"),
    (b"a,b,y\r\n1.5,2,x\r\n3,4,y\r\n", "y", "auto"),
    (b"a,b,y\r1.5,2,x\r3,4,y", "y", "auto"),
    (b"1,2,3\n4,5,6\n", "last", "auto"),
    (b"1,2,3\n4,5,6\n", "0", "auto"),
    (b"1,2,3\n4,5,6\n", "", "auto"),
    (b"1,2,3\n\n\n4,5,6\n\n", "2", "no"),
    (b"x,y\n\"1.5\",\"a\"\"b\"\n\" 2 \",\"c\"\n", "y", "auto"),
    (b"x,y\n\"\",1\n,2\nnan,3\nNA,1\nnull,2\nNuLl,0\n", "y", "auto"),
    (b"x,y\n\"1\"  ,1\n2,1\n", "y", "auto"),
    (b"x,y\n+1e5,1\n-.5,2\n5.,3\n+-7,1\n", "y", "auto"),
    (b"x,y\n1e-46,1\n", "y", "auto"),
    (b"x,y\n7.0064923216240862e-46,1\n3.4028235677973366e38,2\n1.40129846432481707e-45,3\n", "y", "auto"),
    (b"x,y\n3.4028235677973367e38,1\n", "y", "auto"),
    (b"x,y\ninf,1\n", "y", "auto"),
    (b"x,y\n-nan,1\n", "y", "auto"),
    (b"x,y\n1e,1\n", "y", "auto"),
    (b"x,y\n0x10,1\n", "y", "auto"),
    (b"x,y\n1,4294967295\n", "y", "auto"),
    (b"x,y\n1,4294967294\n", "y", "auto"),
    (b"x,y\n1,\n", "y", "auto"),
    (b"x,y\n1,  \n2,a\n", "y", "auto"),
    (b"x,y\n1,cat\n2,dog\n3, cat \n4,\"dog\"\n5,\"a,b\"\n", "y", "auto"),
    (b"x,y\n1,01\n2,1\n", "y", "auto"),
    (b"a,b\n1,\"x\"y\n", "b", "auto"),
    (b"a,b\n1,x\"y\n", "b", "auto"),
    (b"a,b\n1,\"unterminated\n", "b", "auto"),
    (b"", "", "auto"),
    (b"\n\n\r\n", "", "auto"),
    (b"a,b\n1,2,3\n", "", "auto"),
    (b"a,b\n1,2\n", "c", "auto"),
    (b"a,b\n1,2\n", "5", "auto"),
    (b"a,b\n1,2\n", "-1", "auto"),
    (b"a,b\n1,2\n", "b", "maybe"),
    (b"a,b\n1,2\n", "b", "no"),
    (b"a\n1\n", "a", "auto"),
    (b"a,b\n", "b", "auto"),
    (b"1,2\n3,4", "", "yes"),
    (b"1,2\n3,4,", "", "auto"),
    (b"1,2\n3,\n", "", "auto"),
    (b"\"a\"\"b\",c\n1,2\n", "c", "auto"),
    (b"name,\"quoted header\"\n1,2\n", "", "auto"),
    (b"1,2\n3,abc\n", "", "auto"),
    (b"1,2\n3,4\n5,abc\n6,\n", "1", "no"),
    (b"x,y\n" + b"1," + b"9" * 200 + b"\n", "x", "auto"),
    (b"x,y\n0." + b"0" * 60 + b"1,2\n", "y", "auto"),
    (b"x,y\n \t 1.25 \t ,1\n", "y", "auto"),
    (b"\xef\xbb\xbfx,y\n1,2\n", "y", "auto"),
    (b"\xef\xbb\xbfx,y\n1,2\n", "x", "auto"),
    (b"x,y\n\"1\r\n\",1\n2,\"a\r\nb\"\n", "y", "auto"),
    (b"x,y\n\" 2.5\t\",\"lab,el\"\n3,\"lab,el\"\n", "y", "auto"),
    (b"x,y\n1,\"\"\"q\"\"\"\n2,\"\"\"q\"\"\"\n", "y", "auto"),
    (b"a,b,c\n1,2,3\n\"\"\n4,5,6\n", "", "auto"),
    (b"a,b\r\n\r\n1,2\r\n", "", "auto"),
    (b",\n,\n", "", "no"),
]


@needs_ref
@pytest.mark.parametrize("case", range(len(EDGE)))
def test_csv_edge_cases_match_reference(dp, tmp_path, case):
    data, target, header = EDGE[case]
    same(dp, tmp_path, data, target, header)


def random_token(rng: random.Random) -> str:
    k = rng.randrange(10)
    if k == 0:
        b = rng.randrange(0x7f7fffff)
        f = struct.unpack("<f", struct.pack("<I", b))[0]
        return f"{f:.{rng.randrange(6, 12)}e}"
    if k == 1:
        return rng.choice(["", "nan", "NA", "null", " 3 ", "+2", "-0", "1e5", "5.", ".5"])
    if k == 2:
        return str(rng.randrange(-10**12, 10**12)) + "." + str(rng.randrange(10**9))
    if k == 3:
        return f"{rng.gauss(0, 1):.{rng.randrange(1, 20)}f}"
    return f"{rng.uniform(-1e6, 1e6):.{rng.randrange(0, 9)}g}"


@needs_ref
@pytest.mark.parametrize("seed,labels", [(1, "int"), (2, "text"), (3, "int"), (4, "text")])
def test_csv_random_tables_match_reference(dp, tmp_path, seed, labels):
    rng = random.Random(seed)
    rows, cols = rng.randrange(500, 3000), rng.randrange(2, 24)
    eol = rng.choice(["\n", "\r\n", "\r"])
    lines = [",".join(f"f{c}" for c in range(cols)) + ",target"]
    for _ in range(rows):
        cells = [random_token(rng) for _ in range(cols)]
        cells = [f'"{c}"' if rng.random() < 0.05 else c for c in cells]
        lab = str(rng.randrange(7)) if labels == "int" else rng.choice(["alpha", "beta", "gamma", " delta", '"eps"'])
        lines.append(",".join(cells + [lab]))
        if rng.random() < 0.02:
            lines.append("")
    data = (eol.join(lines) + (eol if rng.random() < 0.5 else "")).encode()
    want = same(dp, tmp_path, data, "target", "auto")
    assert "error" not in want and want["rows"] == rows


@needs_ref
def test_csv_large_table_and_training(dp, tmp_path):
    """A 200k x 16 table decoded on the GPU feeds training directly (the
    decoded matrix is the DMatrix's borrowed device input)."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((200_000, 16)).astype(np.float32)
    y = (x[:, 0] + x[:, 1] > 0).astype(np.int64)
    body = "\n".join(",".join(f"{v:.7g}" for v in r) + f",{l}" for r, l in zip(x, y))
    data = (",".join(f"c{i}" for i in range(16)) + ",y\n" + body + "\n").encode()
    same(dp, tmp_path, data, "y", "auto")
    t = dp.CsvTable(data, "y", "auto")
    assert (t.rows, t.features, t.classes) == (200_000, 16, 2)
    import torch
    _, lb = t.to_numpy()
    labels = torch.from_numpy(lb.astype(np.float32)).cuda()
    d = dp.DMatrix(t.values_ptr, t.rows, t.features, label_ptr=labels.data_ptr())
    b = dp.train({"objective": "binary:logistic", "tree_method": "hist", "device": "cuda:0", "max_depth": 4}, d, 3)
    assert b.boosted_rounds() == 3
    b.free()
    d.free()
    t.free()
