"""Generates tests/golden/weights_file_tiny.json from the REFERENCE's own
converter.

Run once in a container that has the reference checkout (not needed at test
time; it does not exist on the GPU hosts):

    python tests/golden/gen_weights_file_golden.py [/path/to/llm-mojo]

What it does
------------
1. Builds the seeded small model of oracle/weights_file.py (TINY_CONFIG,
   30 layers, seed SEED) and writes it as a one-file safetensors checkpoint
   (fp32 tensors, the names convert_gemma4_moe.py:172-232 loads, under
   ``model.language_model.``) in a temporary directory named as the
   converter expects.
2. Runs the reference's ``convert_gemma4_moe.main()`` there, unmodified
   (imported from the reference checkout, cwd = the temporary directory).
   With no embed_tokens / norm tensors in the checkpoint it writes only
   gemma4_moe_weights_q4.bin.
3. Records the file's size and SHA-256, plus the SHA-256 of every 4096-byte
   aligned layer blob as the converter wrote them (cut at the sizes the
   converter's own log reports), in weights_file_tiny.json.

The tests rebuild the same model, write it with the restated writer and
compare hashes, then parse it with the library's layout.
"""
from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import io
import json
import os
import re
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import weights_file as W  # noqa: E402

SEED = 2026
PREFIX = "model.language_model."


def write_safetensors(path: str, tensors: dict):
    """Minimal safetensors writer: 8-byte little-endian header length, JSON
    header of {name: {dtype, shape, data_offsets}}, then the raw data."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        raw = np.ascontiguousarray(arr, np.float32).tobytes()
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def main(ref_root: str):
    cfg = W.TINY_CONFIG
    layers = W.tiny_model(cfg, SEED)
    tensors = {}
    for l, t in enumerate(layers):
        for short, long in W.MATRICES + W.VECTORS:
            if short == "v_proj" and W.is_global(cfg, l):
                continue  # the converter does not load v_proj on global layers
            tensors[f"{PREFIX}layers.{l}.{long}"] = t[short]
    spec = importlib.util.spec_from_file_location("convert_gemma4_moe",
                                                  os.path.join(ref_root, "convert_gemma4_moe.py"))
    conv = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(conv)
    with tempfile.TemporaryDirectory() as tmp:
        model_dir = os.path.join(tmp, "gemma-4-26B-A4B-it-qat-q4_0-unquantized")
        os.makedirs(model_dir)
        write_safetensors(os.path.join(model_dir, "model.safetensors"), tensors)
        cwd = os.getcwd()
        log = io.StringIO()
        try:
            os.chdir(tmp)
            with contextlib.redirect_stdout(log):
                conv.main()
        finally:
            os.chdir(cwd)
        data = open(os.path.join(tmp, "gemma4_moe_weights_q4.bin"), "rb").read()
    sizes = [int(m) for m in re.findall(r"\((\d+) bytes written\)", log.getvalue())]
    assert len(sizes) == cfg["num_layers"] and sum(sizes) == len(data), (sizes, len(data))
    blobs, off = [], 0
    for s in sizes:
        blobs.append(hashlib.sha256(data[off:off + s]).hexdigest())
        off += s
    out = dict(
        generator="convert_gemma4_moe.py (reference, unmodified) on oracle/weights_file.tiny_model",
        config=cfg, seed=SEED, file_bytes=len(data), sha256=hashlib.sha256(data).hexdigest(),
        layer_bytes=sizes, layer_sha256=blobs)
    with open(os.path.join(HERE, "weights_file_tiny.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote weights_file_tiny.json: {len(data)} bytes, sha256 {out['sha256'][:16]}...")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLM_MOJO_REF")
    if not ref:
        sys.exit("usage: gen_weights_file_golden.py /path/to/llm-mojo  (or set LLM_MOJO_REF)")
    main(ref)
