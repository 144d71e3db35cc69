"""Writes the source-manifest header the reference trainer embeds when it is
compiled with DP_TRAIN_SOURCE_MANIFEST (native/class_model_train.cu:6-8,15-17).

Usage: make_ref_manifest.py REF_DIR OUT_HEADER FILE...
       make_ref_manifest.py --json-include   (prints the directory holding
       nlohmann/json.hpp in this Python environment, or nothing)

The manifest maps each compiled reference file to its SHA-256 and pins the
whole map, mirroring the CMake-generated header (CMakeLists.txt:120-145).
"""
import hashlib
import json
import pathlib
import site
import sys
import sysconfig


def json_include() -> str:
    """A directory of this Python environment's site-packages that holds
    nlohmann/json.hpp (the cudnn_frontend wheel ships one)."""
    roots = [sysconfig.get_paths()["purelib"], *site.getsitepackages()]
    for r in roots:
        d = pathlib.Path(r) / "include" / "cudnn_frontend" / "thirdparty"
        if (d / "nlohmann" / "json.hpp").exists():
            return str(d)
    return ""


def main() -> None:
    if sys.argv[1:] == ["--json-include"]:
        print(json_include())
        return
    ref = pathlib.Path(sys.argv[1])
    out = pathlib.Path(sys.argv[2])
    files = {name: hashlib.sha256((ref / name).read_bytes()).hexdigest() for name in sys.argv[3:]}
    files_dump = json.dumps(files, sort_keys=True, separators=(",", ":"))
    manifest = {
        "files": files,
        "sha256": hashlib.sha256(files_dump.encode()).hexdigest(),
        "role": "reference trainer compiled for the drop-in ABI check",
    }
    text = json.dumps(manifest, sort_keys=True, separators=(",", ":"))
    out.write_text(
        "#pragma once\n"
        f"#define DP_TRAIN_SOURCE_MANIFEST_JSON R\"dpmanifest({text})dpmanifest\"\n"
    )


if __name__ == "__main__":
    main()
