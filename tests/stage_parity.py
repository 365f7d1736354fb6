"""Stage-by-stage parity of a compiled, fused executor plan against the CPU
oracle (test infrastructure).

After one run of the graph, the plan is re-executed one step at a time
through the engine's per-step debug interface (icx_engine_step_info /
run_step / value_copy), so fusion stays exactly as the timed plan has it.
Every step's int8 stage is fed its OWN GPU inputs and compared with the
oracle restatement of the reference operators:

* DynamicQuantizeLinear (full, quantise-only after a producer's fused
  (min, max), global): u8 output, scale and zero point bit-exact over the
  whole tensor (dynamic_quantize_linear.rs:32-112);
* QuantLinear / QuantLinear(QKV) / QuantLinear+Residual: the f32 output
  bit-exact on sampled rows (first and last included) - MatMulInteger, Cast,
  Mul, Add and the residual Add each rounded as the reference's CPU
  GraphExecutor does (graph_executor.rs:92-278);
* QuantLinear+GELU: within the GELU tolerance (1e-5 absolute);
* QuantLinear+Residual+LayerNorm: the oracle's exact residual sum put
  through the restated LayerNormalization, within 4e-6 absolute;
* LayerNormalization: on sampled rows against the restated reference
  operator (layer_normalization.rs:25-80) within 4e-6 absolute (the kernel
  sums with a warp tree and multiplies by rsqrt instead of dividing by
  sqrt).
"""
from __future__ import annotations

import numpy as np

from oracle import oracle

GELU_ATOL = 1e-5
LN_ATOL = 4e-6


def sample_rows(M: int, n: int, seed: int = 0) -> np.ndarray:
    if M <= n:
        return np.arange(M)
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(1, M - 1), size=n - 2, replace=False)
    return np.unique(np.concatenate([[0, M - 1], mid]))


def _split(v: str) -> list[str]:
    return v.split("|")


def _weight(inits: dict, name: str) -> np.ndarray:
    """An initializer by name; "<W>#s8" is the engine's exact s8 form of a u8
    weight W (w ^ 0x80, with its zero point converted the same way)."""
    if name.endswith("#s8"):
        return (inits[name[:-3]] ^ np.uint8(0x80)).view(np.int8)
    return inits[name]


def check_plan(ex, inits: dict, rows: int = 64, threads: int = 8, attrs: dict | None = None) -> dict:
    """Re-runs the executor's compiled plan step by step and checks every
    int8 stage against the oracle.  ``inits`` maps initializer names to the
    arrays the graph was built with.  Returns per-kind counts of checked
    steps; raises AssertionError on the first mismatch."""
    counts: dict[str, int] = {}
    for i, (op, node, out, info) in enumerate(ex.steps()):
        if op.startswith("DynamicQuantizeLinear"):
            x = ex.value(info["in"].split(",")[0])
            ex.run_step(i)
            yn, sn, zn = info["outs"].split(",")
            gy, gs, gz = ex.value(yn), ex.value(sn), ex.value(zn)
            ry, rs, rz = oracle.dynamic_quantize_linear(x)
            assert gs.reshape(-1)[0].view(np.uint32) == np.float32(rs).view(np.uint32), \
                f"step {i} {op} {node}: scale {gs.reshape(-1)[0]!r} != {rs!r}"
            assert gz.reshape(-1)[0] == rz, f"step {i} {op} {node}: zero point {gz} != {rz}"
            if not np.array_equal(gy, ry):
                bad = np.argwhere(gy != ry)
                raise AssertionError(f"step {i} {op} {node}: {len(bad)} u8 values differ, "
                                     f"first at {bad[0].tolist()}")
            counts["dql"] = counts.get("dql", 0) + 1
        elif op.startswith("QuantLinear"):
            q = ex.value(info["q"])
            K = q.shape[-1]
            q = q.reshape(-1, K)
            M = q.shape[0]
            s = ex.value(info["s"]).reshape(-1)[0]
            z = ex.value(info["z"]).reshape(-1)[0]
            r = sample_rows(M, rows, seed=i)
            res = ex.value(info["residual"]) if info["residual"] else None
            ex.run_step(i)
            got = ex.value(info["out"])
            got = got.reshape(-1, got.shape[-1])[r]
            gelu = info["gelu"] == "1"
            parts = []
            for w, ws, bias, bz in zip(_split(info["w"]), _split(info["ws"]),
                                       _split(info["bias"]), _split(info["bz"])):
                parts.append(oracle.quant_linear_from_q(
                    q[r], s, z, _weight(inits, w), inits[ws], inits[bias] if bias else None,
                    inits[bz] if bz else None, gelu=gelu, threads=threads))
            ref = np.concatenate(parts, axis=1)
            if res is not None:
                ref = np.add(ref, res.reshape(-1, res.shape[-1])[r], dtype=np.float32)
            if info.get("ln_gamma"):
                # the residual sum is exact; its LayerNorm within LN_ATOL
                ref = oracle.layer_normalization(
                    ref, inits[info["ln_gamma"]],
                    inits[info["ln_beta"]] if info["ln_beta"] else None, float(info["ln_eps"]))
                err = np.abs(got.astype(np.float64) - ref).max()
                assert err <= LN_ATOL, f"step {i} {op} {node}: LayerNorm output off by {err}"
                counts["layernorm"] = counts.get("layernorm", 0) + 1
            elif gelu:
                err = np.abs(got - ref).max()
                assert err <= GELU_ATOL, f"step {i} {op} {node}: GELU output off by {err}"
            elif not np.array_equal(got.view(np.uint32), ref.view(np.uint32)):
                bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
                m, n = bad[0]
                raise AssertionError(
                    f"step {i} {op} {node}: {len(bad)} f32 values differ; row {r[m]} col {n}: "
                    f"{got[m, n]!r} != {ref[m, n]!r}")
            counts[op] = counts.get(op, 0) + 1
        elif op == "LayerNormalization":
            xn, gn, bn = (info["in"].split(",") + ["", ""])[:3]
            x = ex.value(xn)
            D = x.shape[-1]
            x = x.reshape(-1, D)
            r = sample_rows(x.shape[0], rows, seed=i)
            ex.run_step(i)
            got = ex.value(info["outs"].split(",")[0]).reshape(-1, D)[r]
            eps = (attrs or {}).get(node, {}).get("epsilon", 1e-5)
            ref = oracle.layer_normalization(x[r], inits[gn], inits[bn] if bn else None, eps)
            err = np.abs(got.astype(np.float64) - ref).max()
            assert err <= LN_ATOL, f"step {i} {op} {node}: LayerNorm off by {err}"
            counts["layernorm"] = counts.get("layernorm", 0) + 1
        else:
            ex.run_step(i)
            counts["other"] = counts.get("other", 0) + 1
    return counts
