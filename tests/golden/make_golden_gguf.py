"""Generate the GGUF container fixtures in tests/golden/gguf/ and record how the
reference's own parser reads them.

Run (in a checkout that has the reference's sources available):

    python tests/golden/make_golden_gguf.py --reference <path to the reference package sources>

It writes small GGUF files with a writer of its own (every metadata value type,
nested arrays, default and non-default alignment, GGUF versions 2 and 3,
quantized and plain tensors, and malformed variants), imports the reference's
``readers.parse_gguf`` from a throwaway package of symlinks laid out as its
relative imports expect, and stores the parse result (or the exception class
it raised) of every file in ``expected.json``.  Nothing at test time reads the
reference.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "gguf")
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from xanosmerks_b200.synth import make_blocks  # noqa: E402

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def enc_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def enc_value(t, v) -> bytes:
    if t == STR:
        return enc_str(v)
    if t == ARR:
        inner, items = v
        return struct.pack("<IQ", inner, len(items)) + b"".join(enc_value(inner, x) for x in items)
    return struct.pack(_FMT[t], int(v) if t == BOOL else v)


def gguf_bytes(meta, tensors, version=3, alignment=32) -> bytes:
    """meta: [(key, type, value)]; tensors: [(name, dims, type_id, raw bytes)]."""
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(meta))
    for k, t, v in meta:
        head += enc_str(k) + struct.pack("<I", t) + enc_value(t, v)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    for (name, dims, tid, _), o in zip(tensors, offs):
        head += enc_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", tid, o)
    data_start = (len(head) + alignment - 1) // alignment * alignment
    blob = bytearray(head + b"\0" * (data_start - len(head)))
    for (_, _, _, raw), o in zip(tensors, offs):
        blob += b"\0" * (data_start + o - len(blob))
        blob += raw
    return bytes(blob)


def fixtures():
    rng = np.random.default_rng(77)
    q = lambda name, n_blocks: make_blocks(name, n_blocks, rng, "config").tobytes()  # noqa: E731
    meta_a = [("general.architecture", STR, "llama"), ("general.name", STR, "tiny-test"),
              ("t.u8", U8, 200), ("t.i8", I8, -5), ("t.u16", U16, 65000), ("t.i16", I16, -300),
              ("t.u32", U32, 4000000000), ("t.i32", I32, -123456), ("t.f32", F32, 0.15625),
              ("t.bool", BOOL, True), ("t.u64", U64, 2**40 + 3), ("t.i64", I64, -(2**40)), ("t.f64", F64, 1.0 / 3.0),
              ("t.utf8", STR, "Привет, GGUF"), ("t.arr_u8", ARR, (U8, [1, 2, 255])),
              ("t.arr_f32", ARR, (F32, [0.5, -2.25, 1e-3])), ("t.arr_bool", ARR, (BOOL, [True, False, True])),
              ("t.arr_str", ARR, (STR, ["a", "bc", ""])), ("t.arr_nested", ARR, (ARR, [(I32, [1, -2]), (I32, [])])),
              ("t.arr_empty", ARR, (U64, [])), ("llama.block_count", U32, 2)]
    f16 = np.arange(48, dtype=np.float16).tobytes()
    tens_a = [("blk.0.attn_q.weight", [512, 8], 12, q("Q4_K", 16)), ("blk.0.ffn_down.weight", [256, 4], 14, q("Q6_K", 4)),
              ("blk.0.attn_norm.weight", [64], 8, q("Q8_0", 2)), ("token_embd.weight", [16, 3], 1, f16),
              ("output_norm.weight", [10], 0, np.linspace(-1, 1, 10, dtype=np.float32).tobytes()),
              ("rope.bf16", [8, 2], 30, (np.arange(16, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()),
              ("pos.i32", [5], 26, np.arange(5, dtype=np.int32).tobytes()),
              ("blk.1.ffn_up.weight", [256, 2], 13, q("Q5_K", 2)), ("blk.1.ffn_gate.weight", [256, 1], 10, q("Q2_K", 1)),
              ("blk.1.attn_k.weight", [96, 2], 2, q("Q4_0", 6))]
    meta_b = [("general.architecture", STR, "llama"), ("general.alignment", U32, 64)]
    tens_b = [("w", [256, 4], 12, q("Q4_K", 4)), ("b", [7], 0, np.ones(7, np.float32).tobytes())]
    files = {
        "model_a.gguf": gguf_bytes(meta_a, tens_a, version=3),
        "model_b.gguf": gguf_bytes(meta_b, tens_b, version=2, alignment=64),
        "model_iq.gguf": gguf_bytes(meta_b, [("iq", [256], 16, bytes(66))], version=3, alignment=64),
        "bad_magic.gguf": b"GGUX" + gguf_bytes(meta_b, tens_b)[4:],
        "bad_version.gguf": gguf_bytes(meta_b, tens_b, version=6),
        "bad_meta_type.gguf": gguf_bytes([], [])[:24].replace(struct.pack("<Q", 0), struct.pack("<Q", 1), 1)[:16]
        + struct.pack("<QQ", 0, 1) + enc_str("x") + struct.pack("<I", 13) + b"\0" * 8,
        "bad_ndims.gguf": b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + enc_str("t") + struct.pack("<I", 9) + b"\0" * 96,
        "bad_array_len.gguf": b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + enc_str("a") + struct.pack("<IIQ", ARR, U8, 10_000_001),
        "truncated_tensors.gguf": gguf_bytes(meta_b, tens_b)[:-400][: len(gguf_bytes(meta_b, []))],
        "truncated_meta.gguf": gguf_bytes(meta_a, [])[:120],
    }
    return files


def load_reference_parser(ref_dir):
    tmp = tempfile.mkdtemp(prefix="xmref_gguf_")
    pkg = os.path.join(tmp, "xmrefg")
    layout = {"readers.py": "readers.py", "support_tools/core_spr/ref_exceptions.py": "exceptions.py",
              "support_tools/core_spr/dtype_map.py": "dtype_map.py", "support_tools/core_spr/byte_utils.py": "byte_utils.py",
              "support_tools/sup2_spr/path_utils.py": "path_utils.py"}
    for dst, src in layout.items():
        full = os.path.join(pkg, dst)
        os.makedirs(os.path.dirname(full), exist_ok=True)
        os.symlink(os.path.join(ref_dir, src), full)
    # readers.py imports exception classes that the reference's exceptions.py
    # does not define; the shim re-exports the real ones and adds empty classes
    # for the missing names (no parsing logic lives there).
    names = ["InvalidConfigError", "MissingRequiredFieldError", "UnknownArchitectureError", "TokenizerNotFoundError",
             "InvalidTokenizerError", "TokenizerFormatError", "CorruptedSafetensorsError", "CorruptedGGUFError",
             "ShardMismatchError", "ShardIncompleteError", "WeightFormatError"]
    with open(os.path.join(pkg, "support_tools/core_spr/exceptions.py"), "w") as f:
        f.write("from .ref_exceptions import *  # noqa\nfrom . import ref_exceptions as _r\n")
        for nm in names:
            f.write(f"{nm} = getattr(_r, {nm!r}, None) or type({nm!r}, (Exception,), {{}})\n")
    for d in ("", "support_tools", "support_tools/core_spr", "support_tools/sup2_spr"):
        open(os.path.join(pkg, d, "__init__.py"), "w").close()
    sys.path.insert(0, tmp)
    return importlib.import_module("xmrefg.readers")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    readers = load_reference_parser(args.reference)
    os.makedirs(OUT, exist_ok=True)
    expected = {}
    for name, blob in fixtures().items():
        path = os.path.join(OUT, name)
        with open(path, "wb") as f:
            f.write(blob)
        try:
            info = readers.parse_gguf(path)
            info.pop("file")
            expected[name] = {"ok": info}
        except Exception as e:  # noqa: BLE001
            expected[name] = {"error": type(e).__name__}
    with open(os.path.join(OUT, "expected.json"), "w") as f:
        json.dump(expected, f, indent=1, ensure_ascii=False, sort_keys=True)
    print({k: ("ok" if "ok" in v else v["error"]) for k, v in expected.items()})


if __name__ == "__main__":
    main()
