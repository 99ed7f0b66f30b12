"""Generate the golden fixtures in this directory from the reference's own oracle.

Run in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_golden.py /path/to/algebraic-intelligence

The script imports ``tests/reference_attention.py`` and ``tests/reference_ago.py``
of the reference (pure NumPy, float64) *read-only* from the given checkout and
evaluates them on the seeded inputs of ``inputs.py``; the attention fixtures go
to ``golden.npz``, the AGO rotation fixtures to ``golden_ago.npz``. The reference's own tests seed with JAX PRNG keys,
which cannot be regenerated without JAX, so NumPy ``default_rng`` seeds are used
instead. Inputs are not stored; their SHA-256 is, and the tests regenerate them
and check the digest. Small outputs are stored in float64; the two larger ones
(config 1 and L=180) in float32, which is ample for the 1e-5 parity bar they
serve. Nothing at test time reads the reference checkout.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import inputs  # noqa: E402


def _load_reference_oracle(root: Path, name: str = "reference_attention.py"):
    path = root / "tests" / name
    spec = importlib.util.spec_from_file_location("_ref_oracle_" + name.split(".")[0], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, path


AGO_TABLE_ROWS = [0, 1, 2, 3, 127, 128, 1000, 4095]


def make_ago(root: Path) -> None:
    """AGO tables and rotations from tests/reference_ago.py."""
    ref, path = _load_reference_oracle(root, "reference_ago.py")
    out, digests = {}, {}
    c, s = ref.build_cayley_rotary_matrix_fp64(32, 64)
    out["table_d32_l64_c"], out["table_d32_l64_s"] = c, s
    c, s = ref.build_cayley_rotary_matrix_fp64(128, 4096)
    out["table_d128_l4096_rows_c"], out["table_d128_l4096_rows_s"] = c[AGO_TABLE_ROWS], s[AGO_TABLE_ROWS]
    freqs = np.array([0.9, 0.5, 0.1, 0.01])
    c, s = ref.build_cayley_rotary_matrix_fp64(8, 16, freqs=freqs)
    out["table_d8_l16_freqs_c"], out["table_d8_l16_freqs_s"] = c, s
    c, s = ref.build_cayley_rotary_matrix_fp64(16, 8, base=500.0)
    out["table_d16_l8_base500_c"], out["table_d16_l8_base500_s"] = c, s
    q, k = inputs.ago_small()
    digests["ago_small"] = inputs.digest(q, k)
    out["ago_small_q"], out["ago_small_k"] = ref.apply_ago_rotations_fp64(q, k)
    q, k = inputs.ago_bhtd()
    digests["ago_bhtd"] = inputs.digest(q, k)
    out["ago_bhtd_q"], out["ago_bhtd_k"] = ref.apply_ago_rotations_fp64(q, k, seq_axis=2)
    np.savez_compressed(HERE / "golden_ago.npz", **out)
    meta = {
        "generator": "tests/golden/make_golden.py",
        "reference_file": "tests/reference_ago.py",
        "reference_file_sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
        "numpy": np.__version__,
        "input_sha256": digests,
        "table_d128_l4096_rows": AGO_TABLE_ROWS,
        "keys": sorted(out),
    }
    (HERE / "golden_ago_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(out)} arrays to {HERE / 'golden_ago.npz'}")


def main(root: str) -> None:
    ref, path = _load_reference_oracle(Path(root))
    out = {}
    digests = {}

    x = inputs.octic_grid()
    digests["octic_grid"] = inputs.digest(x)
    out["octic_y"] = ref.kernel(x)

    x = inputs.softmax_rows()
    digests["softmax_rows"] = inputs.digest(x)
    for sink in (0.0, 0.5, 1.0):
        out[f"asm_y_sink{sink}"] = ref.attention(x, sink)

    x = inputs.softmax_long_rows()
    digests["softmax_long_rows"] = inputs.digest(x)
    out["asm_long_y"] = ref.attention(x, 0.5).astype(np.float32)

    q, k, v = inputs.afa_small()
    digests["afa_small"] = inputs.digest(q, k, v)
    out["afa_small_y"] = ref.reference_afa(q, k, v, sink=0.5, causal=False)
    out["afa_small_y_causal"] = ref.reference_afa(q, k, v, sink=0.5, causal=True)

    q, k, v = inputs.afa_l180()
    digests["afa_l180"] = inputs.digest(q, k, v)
    out["afa_l180_y"] = ref.reference_afa(q, k, v, sink=0.5, causal=False).astype(np.float32)
    out["afa_l180_y_causal"] = ref.reference_afa(q, k, v, sink=0.5, causal=True).astype(np.float32)

    q, k, v = inputs.config1()
    digests["config1"] = inputs.digest(q, k, v)
    d = q.shape[-1]
    s = np.matmul(q.astype(np.float64), np.swapaxes(k.astype(np.float64), -1, -2)) / np.sqrt(d)
    out["cfg1_softmax_o"] = np.matmul(ref.attention(s, 0.5, 1e-5), v.astype(np.float64)).astype(np.float32)
    out["cfg1_afa_o"] = ref.reference_afa(q, k, v, sink=0.5, causal=False).astype(np.float32)

    x, g, xl, gl = inputs.softmax_vjp()
    digests["softmax_vjp"] = inputs.digest(x, g, xl, gl)
    for sink in (0.0, 0.5, 1.0):
        out[f"asm_vjp_sink{sink}"] = ref.attention_vjp(x, g, sink)
    out["asm_vjp_long"] = ref.attention_vjp(xl, gl, 0.5)

    q, k, v = inputs.decode_small()
    digests["decode_small"] = inputs.digest(q, k, v)
    out["dec_y"] = ref.reference_afa(q, k, v, sink=0.5, causal=False)

    np.savez_compressed(HERE / "golden.npz", **out)
    meta = {
        "generator": "tests/golden/make_golden.py",
        "reference_file": "tests/reference_attention.py",
        "reference_file_sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
        "numpy": np.__version__,
        "input_sha256": digests,
        "keys": sorted(out),
    }
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(out)} arrays to {HERE / 'golden.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to a checkout of the reference repository>")
    root = sys.argv[1]
    main(root)
    make_ago(Path(root))
