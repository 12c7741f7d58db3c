"""Generate golden fixtures by executing the reference's own CPU functions.

Run where the reference source tree is checked out, naming its root (the directory that holds
``src/lib/webgpu/kernels.ts``) as the argument or in ``$BRK_REFERENCE``:

    python tests/golden/gen_golden.py <path-to-Brimkern-checkout>

It extracts ``attentionCpu``, ``ropeCpu``, ``ropeFactorsCpu`` and ``rmsnormCpu`` verbatim from
``src/lib/webgpu/kernels.ts`` (lines 3395-3495), and the inline reference loop of the
attention_full gate (kernels.ts:3171-3177, wrapped in a function that declares its inputs), runs
them through ``jsmini`` (a JS-subset interpreter with JS number semantics; no JavaScript engine
exists in this image) on seeded inputs, and writes ``golden.npz`` + ``golden.json`` next to this
file.  The cases replay the reference's own selfValidate shapes (kernels.ts:2519-2535, 2556-2568,
2611-2640, 3168-3201), the QK-norm shape of the Qwen3 gate (kernels.ts:2676-2688) and the
config-1 decode shape.
The fixtures are committed; tests read them without the reference.
"""
from __future__ import annotations

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import jsmini  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BRK_REFERENCE", "")
KERNELS_TS = os.path.join(REF, "src", "lib", "webgpu", "kernels.ts")
FUNCS = ["rmsnormCpu", "ropeFactorsCpu", "ropeCpu", "attentionCpu"]


def uniform(rng, n):
    """Math.random() * 2 - 1, as the reference's rand() (kernels.ts:2265), but seeded."""
    return (rng.random(n) * 2 - 1).astype(np.float32)


def normal(rng, n):
    return rng.standard_normal(n).astype(np.float32)


def cases():
    out = []
    rng = np.random.default_rng(20261201)
    # --- RoPE gates (kernels.ts:2519-2535)
    out.append(dict(name="rope_small", fn="ropeCpu", rows=2, head_dim=4, n_heads=2, past_len=1, base=10000.0,
                    x=uniform(rng, 2 * 4)))
    x = uniform(rng, 6 * 64)
    out.append(dict(name="rope_ff_ones", fn="ropeFactorsCpu", rows=6, head_dim=64, n_heads=2, past_len=7,
                    base=500000.0, x=x, ff=np.ones(32, np.float32)))
    out.append(dict(name="rope_ff_plain", fn="ropeCpu", rows=6, head_dim=64, n_heads=2, past_len=7, base=500000.0, x=x))
    ff = np.array([1 + (i % 5) * 0.7 for i in range(32)], np.float32)
    out.append(dict(name="rope_ff_distinct", fn="ropeFactorsCpu", rows=6, head_dim=64, n_heads=2, past_len=7,
                    base=500000.0, x=x, ff=ff))
    # Qwen3 decode shape, large position (theta 1e6, pos 4095), and Llama-3.2 long position (pos 131071).
    out.append(dict(name="rope_qwen3_pos4095", fn="ropeCpu", rows=8, head_dim=128, n_heads=8, past_len=4095,
                    base=1e6, x=normal(rng, 8 * 128)))
    out.append(dict(name="rope_llama_pos131071", fn="ropeFactorsCpu", rows=8, head_dim=64, n_heads=8,
                    past_len=131071, base=500000.0, x=normal(rng, 8 * 64),
                    ff=np.array([1 + (i % 7) * 4.5 for i in range(32)], np.float32)))
    # --- per-head RMSNorm (QK-norm) as used at kernels.ts:1707-1709
    out.append(dict(name="rmsnorm_qk_small", fn="rmsnormCpu", rows=12, dim=4, eps=1e-6, one_plus=False,
                    x=uniform(rng, 48), w=uniform(rng, 4)))
    out.append(dict(name="rmsnorm_qk_hd128", fn="rmsnormCpu", rows=8, dim=128, eps=1e-6, one_plus=False,
                    x=normal(rng, 8 * 128), w=(1 + 0.02 * rng.standard_normal(128)).astype(np.float32)))
    out.append(dict(name="rmsnorm_oneplus", fn="rmsnormCpu", rows=4, dim=256, eps=1e-6, one_plus=True,
                    x=normal(rng, 4 * 256), w=(0.1 * rng.standard_normal(256)).astype(np.float32)))
    out.append(dict(name="rmsnorm_default_eps", fn="rmsnormCpu", rows=3, dim=64, eps=None, one_plus=None,
                    x=normal(rng, 3 * 64), w=normal(rng, 64)))

    # --- attention gates (kernels.ts:2556-2568, 2611-2640)
    def att(name, nT, nH, nKv, hd, past, scale=None, softcap=None, dist=uniform):
        kv = past + nT
        out.append(dict(name=name, fn="attentionCpu", n_tokens=nT, n_heads=nH, n_kv_heads=nKv, head_dim=hd,
                        past_len=past, scale=scale, softcap=softcap, q=dist(rng, nT * nH * hd),
                        k=dist(rng, kv * nKv * hd), v=dist(rng, kv * nKv * hd)))

    att("att_gqa_plain", 2, 4, 2, 4, 2)
    att("att_gqa_softcap", 2, 4, 2, 4, 2, scale=0.3, softcap=5.0)
    att("att_decode_qwen05_past300", 1, 14, 2, 64, 300)
    att("att_decode_qwen05_nt10_past173", 10, 14, 2, 64, 173)
    att("att_decode_softcap_hd8", 2, 4, 2, 8, 173, scale=0.3, softcap=5.0)
    att("att_decode_hd128_past70", 1, 2, 1, 128, 70)
    att("att_decode_hd256_gemma", 1, 8, 4, 256, 40, scale=1 / 16, softcap=50.0, dist=normal)
    att("att_prefill_past0", 7, 4, 2, 16, 0, dist=normal)
    # config 1: Qwen2.5-0.5B decode, positions 0..1023 + 1 new token, N(0,1), scale 1/8 (default)
    att("att_config1_qwen05_past1024", 1, 14, 2, 64, 1024, dist=normal)

    # --- non-causal attention_full gates (kernels.ts:3168-3201): the cross-attention shape, then
    # the UNet shapes of the workgroup-kernel gate (partial tile, CLIP text length, head_dim 160).
    def full(name, nT, kvL, nH, hd, dist=uniform):
        out.append(dict(name=name, fn="attentionFullGate", n_tokens=nT, kv_len=kvL, n_heads=nH, head_dim=hd,
                        q=dist(rng, nT * nH * hd), k=dist(rng, kvL * nH * hd), v=dist(rng, kvL * nH * hd)))

    full("full_gate_cross", 3, 5, 2, 4)
    full("full_sdturbo_self", 70, 70, 5, 64)
    full("full_clip_cross", 16, 77, 5, 64)
    full("full_sdxs_hd160", 9, 9, 8, 160)
    return out


def extract_full_gate(src: str) -> str:
    """The attention_full gate's reference loop (kernels.ts:3171-3177), verbatim, inside a function
    that declares the names it uses (the gate's own declarations at kernels.ts:3170)."""
    marker = src.index("// attention_full: NON-causal")
    start = src.index("for (let h = 0; h < nH; h++) for (let t = 0; t < nT; t++) {", marker)
    end = src.index("if (!closeRel(await this.attentionFull(aq, ak, av", start)
    body = src[start:end].rstrip()
    return ("function attentionFullGate(aq, ak, av, nT, kvL, nH, hd2) {\n"
            "const dd = nH * hd2, sc = 1 / Math.sqrt(hd2);\n"
            "const aref = new Float32Array(nT * dd);\n" + body + "\nreturn aref;\n}")


def run_case(interp, c):
    fn = c["fn"]
    if fn == "ropeCpu":
        r = interp.call(fn, jsmini.F32Array(c["x"]), float(c["rows"]), float(c["head_dim"]), float(c["n_heads"]),
                        float(c["past_len"]), float(c["base"]))
    elif fn == "ropeFactorsCpu":
        r = interp.call(fn, jsmini.F32Array(c["x"]), jsmini.F32Array(c["ff"]), float(c["rows"]), float(c["head_dim"]),
                        float(c["n_heads"]), float(c["past_len"]), float(c["base"]))
    elif fn == "rmsnormCpu":
        args = [jsmini.F32Array(c["x"]), jsmini.F32Array(c["w"]), float(c["rows"]), float(c["dim"])]
        if c["eps"] is not None:
            args.append(float(c["eps"]))
            if c["one_plus"] is not None:
                args.append(bool(c["one_plus"]))
        r = interp.call(fn, *args)
    elif fn == "attentionFullGate":
        r = interp.call(fn, jsmini.F32Array(c["q"]), jsmini.F32Array(c["k"]), jsmini.F32Array(c["v"]),
                        float(c["n_tokens"]), float(c["kv_len"]), float(c["n_heads"]), float(c["head_dim"]))
    elif fn == "attentionCpu":
        args = [jsmini.F32Array(c["q"]), jsmini.F32Array(c["k"]), jsmini.F32Array(c["v"]), float(c["n_tokens"]),
                float(c["n_heads"]), float(c["n_kv_heads"]), float(c["head_dim"]), float(c["past_len"])]
        if c["scale"] is not None or c["softcap"] is not None:
            args.append(jsmini.UNDEF if c["scale"] is None else float(c["scale"]))
        if c["softcap"] is not None:
            args.append(float(c["softcap"]))
        r = interp.call(fn, *args)
    else:
        raise KeyError(fn)
    return r.a.copy()


def main():
    if not REF or not os.path.isfile(KERNELS_TS):
        sys.exit("usage: gen_golden.py <Brimkern checkout> (or set BRK_REFERENCE); "
                 f"no src/lib/webgpu/kernels.ts under {REF!r}")
    src = open(KERNELS_TS, encoding="utf-8").read()
    interp = jsmini.Interpreter()
    for f in FUNCS:
        interp.load(jsmini.extract_function(src, f))
    interp.load(extract_full_gate(src))
    arrays, manifest = {}, []
    for c in cases():
        t0 = time.time()
        out = run_case(interp, c)
        meta = {k: v for k, v in c.items() if not isinstance(v, np.ndarray)}
        for k, v in c.items():
            if isinstance(v, np.ndarray):
                arrays[f"{c['name']}/{k}"] = v
        arrays[f"{c['name']}/out"] = out
        manifest.append(meta)
        print(f"{c['name']:34s} {out.size:7d} values  {time.time() - t0:6.1f}s", flush=True)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as fh:
        json.dump({"source": "src/lib/webgpu/kernels.ts:3395-3495 and 3171-3177 executed by tests/golden/jsmini.py",
                   "cases": manifest}, fh, indent=1)


if __name__ == "__main__":
    main()
