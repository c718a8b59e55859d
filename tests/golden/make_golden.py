"""Generate golden vectors by executing the reference's own pure-Python restatement.

The reference ships an independent pure-Python reading of its BF16 perturbation
in ``ops/bf16_parity.py:18-106`` (mix64, sign, decode, encode, next_value,
cpu_values).  That module imports ``jax`` at top level and jax is absent here, so
this script parses the file with ``ast``, keeps only those pure functions (and
the ``MASK64`` constant) and executes them.  Their outputs become the committed
fixture ``bf16_parity.json``; the C oracle and the CUDA path are both checked
against it, which pins the oracle to the reference's own arithmetic.

Run from the repository root (needs the reference checkout; the fixture it
writes is committed so the GPU box never needs the reference):

    python tests/golden/make_golden.py /path/to/ennx-reference
"""
from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

import numpy as np

KEEP = {"f32", "mix64", "sign", "decode", "encode", "next_value", "cpu_values"}


def load_reference_functions(ref_root: Path) -> dict:
    src = (ref_root / "ops" / "bf16_parity.py").read_text()
    tree = ast.parse(src)
    body = [ast.Import(names=[ast.alias(name="math")]), ast.Import(names=[ast.alias(name="struct")])]
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in KEEP:
            body.append(node)
        elif isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id in ("MASK64", "MAX_F32") for t in node.targets
        ):
            body.append(node)
    module = ast.Module(body=body, type_ignores=[])
    ast.fix_missing_locations(module)
    ns: dict = {}
    exec(compile(module, "bf16_parity_pure", "exec"), ns)
    missing = KEEP - set(ns)
    if missing:
        raise SystemExit(f"reference functions not found: {sorted(missing)}")
    return ns


def bf16_bits(x: np.ndarray) -> np.ndarray:
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path to the Kvutza/ennx checkout>")
    ref_root = Path(sys.argv[1])
    ns = load_reference_functions(ref_root)
    out_dir = Path(__file__).resolve().parent

    cases = []
    # Case 1: the hardware parity case of ops/bf16_parity.py:393-418 (size
    # 1030, linspace(-4, 4) with +0/-0 at [0, 1], three leaves, three terms).
    # jax.numpy.linspace in bf16 is not available here; the base is the
    # float32 linspace rounded to bf16 (it is an input, not a result).
    size = 1030
    base = bf16_bits(np.linspace(-4.0, 4.0, size, dtype=np.float32))
    base[0] = 0x0000
    base[1] = 0x8000
    leaves = [(17, 0, 257, 1.0e-6), (19, 257, 516, 1.0e-3), (23, 773, 257, 0.25)]
    terms = [(41, 0.25), (73, -0.125), (89, 0.03125)]
    cases.append({"name": "bf16_parity_main", "base": base.tolist(), "leaves": leaves,
                  "terms": terms, "expected": ns["cpu_values"](base.tolist(), leaves, terms)})

    # Case 2: adversarial shapes in the spirit of docs/testing.md (powers of
    # two +- 1, limits, zeros, a single term, a cancelling pair plus a third).
    rng = np.random.default_rng(7)
    for n in (1, 31, 33, 255, 257):
        vals = rng.standard_normal(n).astype(np.float32) * np.float32(3.0)
        b = bf16_bits(vals)
        if n >= 4:
            b[:4] = [0x0000, 0x8000, 0x7F7F, 0xFF7F]
        split = max(1, n // 3)
        lv = [(1000 + n, 0, split, 1.0e-3)]
        if n - split > 0:
            lv.append((2000 + n, split, n - split, 0.5))
        tm = [(0x123456789ABCDEF0, 0.5), (91, -0.125), (91, 0.0625)] if n % 2 else [(5, 1.0)]
        cases.append({"name": f"bf16_adversarial_{n}", "base": b.tolist(), "leaves": lv,
                      "terms": tm, "expected": ns["cpu_values"](b.tolist(), lv, tm)})

    signs = [ns["sign"](0x123456789ABCDEF0, 11, e) for e in range(64)]
    mixes = [ns["mix64"](v) for v in (0, 1, 2**63, 2**64 - 1, 0x0123456789ABCDEF)]
    payload = {
        "generator": "tests/golden/make_golden.py (executes ops/bf16_parity.py:18-106 of the reference)",
        "cases": cases,
        "signs_seed_0x123456789abcdef0_key_11": signs,
        "mix64": {"inputs": [0, 1, 2**63, 2**64 - 1, 0x0123456789ABCDEF], "outputs": mixes},
    }
    (out_dir / "bf16_parity.json").write_text(json.dumps(payload))
    print(f"wrote {out_dir / 'bf16_parity.json'}: {len(cases)} cases")


if __name__ == "__main__":
    main()
