"""Regenerates the committed golden fixtures from the reference checkout.

Run in a container that has the reference tree (read-only) and torch/numpy/gguf:

    python tests/golden/make_golden.py /path/to/reference

Outputs (small, committed):
  selftest_hashes.json  sha256 of every stored tensor of the reference's in-container quantizer
                        self-test (`modal/results/2026-11-09-weight-error-selftest-container.json`,
                        produced by `modal/weight_error_app.py:472-510`).
  gguf_golden.npz       the ggml-quantized Q8_0 / Q4_K bytes of the two 96x1024 self-test cases
                        (base64 fields of that JSON); their decoded sha256 is in the JSON file.
  kitchen_w4a8.npz      the W4A8 (fitted/fixed codebook) and W6A8 stored tensors of the
                        gauss_96x1024 case, plus the int8 grid and fp32 weight that the
                        reference's own CPU port (`dequantize_w4a8`, `modal/weight_error_app.py:326`)
                        decodes them to, run here.

Nothing at test time reads the reference tree; tests read only these files.
"""
import base64
import hashlib
import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_port(ref_root):
    """Import modal/weight_error_app.py with a stub `modal` module (the same stub the reference's
    own validator uses, `modal/weight_error_validate.py:29-42`)."""
    stub = types.ModuleType("modal")

    class _Any:
        def __call__(self, *a, **k):
            return a[0] if len(a) == 1 and callable(a[0]) and not k else self

        def __getattr__(self, name):
            return self

    stub.App = stub.Volume = stub.Image = _Any()
    sys.modules["modal"] = stub
    spec = importlib.util.spec_from_file_location("weight_error_app", os.path.join(ref_root, "modal", "weight_error_app.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root):
    src = os.path.join(ref_root, "modal", "results", "2026-11-09-weight-error-selftest-container.json")
    data = json.load(open(src))
    hashes = {"source": "modal/results/2026-11-09-weight-error-selftest-container.json",
              "torch": data.get("torch"), "gguf": data.get("gguf"), "cases": {}}
    gguf_arrays = {}
    for case, entry in data["cases"].items():
        out = {"input_sha256": entry["input_sha256"], "formats": {}}
        for fmt, f in entry["formats"].items():
            out["formats"][fmt] = {k: v for k, v in f.items()
                                   if isinstance(v, str) and not k.endswith("_b64")}
            if fmt.startswith("gguf_") and "q_b64" in f:
                gguf_arrays[f"{case}__{fmt}"] = np.frombuffer(base64.b64decode(f["q_b64"]), dtype=np.uint8)
        hashes["cases"][case] = out
    with open(os.path.join(HERE, "selftest_hashes.json"), "w") as fh:
        json.dump(hashes, fh, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "gguf_golden.npz"), **gguf_arrays)

    # Kitchen W4A8 / W6A8: stored tensors of the gauss case and the port's decode of them.
    import torch

    port = load_reference_port(ref_root)
    f = data["cases"]["gauss_96x1024"]["formats"]
    arrays = {}
    for fmt, bits in (("w4a8", 4), ("w6a8", 6)):
        q = np.frombuffer(base64.b64decode(f[fmt]["q_b64"]), dtype=np.int8).reshape(96, -1)
        s_rel = np.frombuffer(base64.b64decode(f[fmt]["s_rel_b64"]), dtype=np.uint8).reshape(96, -1)
        s_ch = np.frombuffer(base64.b64decode(f[fmt]["s_channel_b64"]), dtype=np.float32)
        cb = None
        if "codebook_b64" in f[fmt]:
            cb = np.frombuffer(base64.b64decode(f[fmt]["codebook_b64"]), dtype=np.float32)
        for name, arr in (("q", q), ("s_rel", s_rel), ("s_channel", s_ch)):
            assert hashlib.sha256(arr.tobytes()).hexdigest() == f[fmt][name], (fmt, name)
        qt = torch.from_numpy(q.copy())
        st = torch.from_numpy(s_rel.copy()).view(torch.float8_e4m3fn)
        ct = torch.from_numpy(s_ch.copy())
        cbt = None if cb is None else torch.from_numpy(cb.copy())
        k = 1024
        codes = port._unpack_codes(qt, k, bits)
        values = cbt[codes] if cbt is not None else codes.float() - float(1 << (bits - 1))
        grid = (values.view(96, k // 16, 16) * st.float().unsqueeze(-1)).view(96, k).round().clamp_(-127, 127).to(torch.int8)
        deq = port.dequantize_w4a8(qt, st, ct, cbt)
        arrays[f"{fmt}_q"] = q
        arrays[f"{fmt}_s_rel"] = s_rel
        arrays[f"{fmt}_s_channel"] = s_ch
        if cb is not None:
            arrays[f"{fmt}_codebook"] = cb
        arrays[f"{fmt}_grid"] = grid.numpy()
        arrays[f"{fmt}_deq16"] = deq.numpy().astype(np.float32)[:16]  # first 16 rows keep the file small
    np.savez_compressed(os.path.join(HERE, "kitchen_w4a8.npz"), **arrays)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QLIN_REFERENCE", "."))
