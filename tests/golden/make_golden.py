"""Generate the golden vectors that pin the oracle to the reference.

Run in a container where the DeepUnity reference is checked out, naming its
project root in DU_REFERENCE (required; there is no default path):

    DU_REFERENCE=<project root> python tests/golden/make_golden.py

It writes, next to this script:
  quant_golden.npz   seeded fp32 matrices and what the reference's own
                     quantize_int8 / quantize_int4 (import_params.py:229-248)
                     return for them -- int4 at the reference's G4 = 32 and at
                     G = 128 (the same function with its module-level G4 set
                     to 128), including edge rows (all zeros, ties, tiny values,
                     a row whose max is negative, a row of +/- equal extremes);
  int8_export.npz    the first 32 rows of a real `import_params.py --quant int8`
                     export shipped with the reference
                     (Assets/Resources/Weights/weights_qwen3.5_0.8B_roleplay_1308_int8/
                      layer_3/mlp_down_proj.int8.bin, 1024 x 3584 int8, + .scales.bin),
                     the dequantised values numpy computes for them, and
                     checksums of the whole file;
  f16_golden.npz     numpy float32 -> float16 rounding of edge values.
Nothing at test time reads the reference; the tests read only these files.
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("DU_REFERENCE", "")
IMP_PATH = os.path.join(REF, "Assets/DeepUnity/InferenceEngine/import_params.py")
EXPORT = os.path.join(REF, "Assets/Resources/Weights/weights_qwen3.5_0.8B_roleplay_1308_int8/layer_3")


def require_reference():
    if not REF or not os.path.isfile(IMP_PATH):
        sys.exit("make_golden.py: set DU_REFERENCE to the DeepUnity project root "
                 "(the directory holding Assets/DeepUnity/InferenceEngine/import_params.py)")


def load_imp():
    spec = importlib.util.spec_from_file_location("du_import_params", IMP_PATH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def edge_rows(cols):
    rows = [np.zeros(cols, np.float32)]                       # all zeros -> 1e-8 / 1e-10 floor
    r = np.zeros(cols, np.float32); r[::7] = 0.5; r[3] = -0.5  # ties between +/- extremes
    rows.append(r)
    rows.append(np.full(cols, 1e-12, np.float32))              # below the int4 d floor
    r = np.linspace(-1.0, 0.25, cols, dtype=np.float32)        # negative max magnitude
    rows.append(r)
    r = np.zeros(cols, np.float32); r[5] = 3.0; r[6] = -3.0    # equal |max| of opposite sign
    rows.append(r)
    r = (np.arange(cols, dtype=np.float32) - cols / 2) * 0.03125  # exact half steps -> rint ties
    rows.append(r)
    return np.stack(rows)


def main():
    require_reference()
    imp = load_imp()
    rng = np.random.default_rng(0)
    out = {}
    for name, (rows, cols) in {"a": (64, 256), "b": (37, 384), "c": (8, 1024)}.items():
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        w = np.concatenate([w, edge_rows(cols)], axis=0)
        out[f"{name}_w"] = w
        q8, s8, _ = imp.quantize_int8(w)
        out[f"{name}_q8"], out[f"{name}_s8"] = q8, s8.view(np.uint16)
        imp.G4 = 32
        p4, d4, _ = imp.quantize_int4(w)
        out[f"{name}_p4_g32"], out[f"{name}_d4_g32"] = p4, d4.view(np.uint16)
        imp.G4 = 128
        p4, d4, _ = imp.quantize_int4(w)
        out[f"{name}_p4_g128"], out[f"{name}_d4_g128"] = p4, d4.view(np.uint16)
        imp.G4 = 32
    # config-1 matrix: W fp32 [1024, 1024] ~ N(0, 0.02), x ~ N(0, 1), seed 0
    rng = np.random.default_rng(0)
    x1 = rng.standard_normal((1, 1024)).astype(np.float32)
    w1 = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    q1, s1, _ = imp.quantize_int8(w1)
    # the matrix is regenerated from the seed at test time; only digests of the
    # reference's quantized bytes and the first rows are stored
    out["c1_x"], out["c1_q8_head"], out["c1_s8"] = x1, q1[:16], s1.view(np.uint16)
    out["c1_q8_sha256"] = np.frombuffer(hashlib.sha256(q1.tobytes()).digest(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)

    q = np.fromfile(os.path.join(EXPORT, "mlp_down_proj.int8.bin"), dtype=np.int8).reshape(1024, 3584)
    s = np.fromfile(os.path.join(EXPORT, "mlp_down_proj.scales.bin"), dtype=np.float16)
    raw = open(os.path.join(EXPORT, "mlp_down_proj.int8.bin"), "rb").read()
    deq = q[:32].astype(np.float32) * s[:32, None].astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "int8_export.npz"), q=q[:32], s=s[:32].view(np.uint16), deq=deq,
                        sha256=np.frombuffer(hashlib.sha256(raw).digest(), np.uint8),
                        row_absmax=np.abs(q.astype(np.int32)).max(axis=1).astype(np.int32),
                        row_sum=q.astype(np.int64).sum(axis=1), shape=np.array([1024, 3584]))

    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 65519.99, 1e6, 6.1035156e-05, 6.0e-05,
                     5.9604645e-08, 2.98e-08, 2.9802322e-08, 1e-8, 0.1, 0.2, 1.0009765625, 1.00048828125,
                     1.000732421875, 3.14159265, np.inf, -np.inf], np.float32)
    rnd = np.concatenate([rng.standard_normal(4096).astype(np.float32) * s_ for s_ in (1e-6, 1e-3, 1.0, 1e3)])
    vals = np.concatenate([edge, rnd])
    with np.errstate(over="ignore"):
        h = vals.astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "f16_golden.npz"), x=vals, h=h)
    print("wrote golden vectors to", HERE)


if __name__ == "__main__":
    sys.exit(main())
