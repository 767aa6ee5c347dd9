"""Generate the committed golden vectors under ``tests/golden/``.

Run from the repository root with the reference tree (szibis/MLX-Flash
0.8.0) named by ``$MLXFLASH_REF`` or by the first argument:

    MLXFLASH_REF=/path/to/MLX-Flash python tests/golden/gen_golden.py
    python tests/golden/gen_golden.py /path/to/MLX-Flash
    python tests/golden/gen_golden.py --affine-only     # affine.npz alone

What each fixture pins:

* ``kv_sym.npz`` -- outputs of the reference's OWN ``quantize_tensor`` and
  ``dequantize_tensor`` (``mlx_flash_compress/quantized_kv_cache.py:68-234``),
  executed from the reference source with the NumPy stand-in for ``mlx.core``
  in ``_mlx_standin/`` (MLX itself cannot be installed here).  The script also
  checks that ``oracle.kv_sym`` reproduces every byte, scale and float.
* ``mixed2bit.npz`` -- outputs of the reference's ``requantize_4bit_to_2bit`` /
  ``dequantize_2bit`` (``mlx_flash_compress/mixed_precision.py:130-255``, pure
  NumPy, executed unmodified) on weights packed by ``oracle.affine``.  The
  script checks that ``oracle.mixed`` (which unpacks with ``oracle.affine``)
  matches them bit for bit, which pins the affine unpack order and dequant.
* ``affine.npz`` -- oracle-derived vectors for the affine quantizer (MLX's
  edge rule under ``mlx/``, restated from ml-explore/mlx's ``affine_quantize``;
  the min/max rule elsewhere) and quantized matmul (see ``oracle/affine.py``).
* ``ep_shard.json`` -- ``ExpertShard`` ownership and ``owner_of`` from
  ``mlx_flash_compress/distributed_experts.py:36-80`` executed unmodified.
* ``moe_dispatch.npz`` -- ``moe_dispatch_numpy`` (``kernels/ops.py:138-148``).
* ``kv_evict.npz`` -- the reference's own ``CompressedKVCache`` (H2O and
  ScissorHands scoring, ``kv_compression.py``) and ``StreamingLLMCache``
  (``streaming_llm.py``) executed with the NumPy ``mlx.core`` stand-in on
  seeded update sequences: every step's inputs, the cache contents after the
  step, and the tracked importance arrays.
"""

import importlib.util
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
_ARGS = [a for a in sys.argv[1:] if not a.startswith("--")]
REF = _ARGS[0] if _ARGS else os.environ.get("MLXFLASH_REF")
sys.path.insert(0, ROOT)

from oracle import affine, kv_sym, mixed  # noqa: E402
from oracle.fp import round_to  # noqa: E402


def _load_ref_module(name, relpath, extra_path=None):
    if not REF or not os.path.isdir(REF):
        sys.exit("gen_golden.py needs the reference tree: set MLXFLASH_REF or pass its path as the first argument")
    if extra_path:
        sys.path.insert(0, extra_path)
    path = os.path.join(REF, relpath)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def kv_cases():
    rng = np.random.default_rng(20260101)
    cases = []

    def add(name, x, bits, gs, dtype):
        cases.append((name, round_to(np.asarray(x, np.float32), dtype), bits, gs, dtype))

    for dtype in ("bf16", "f32", "f16"):
        for bits in (2, 4, 8):
            add(f"normal128_{dtype}_b{bits}", rng.standard_normal(128), bits, 64, dtype)
            add(f"kv3d_{dtype}_b{bits}", rng.standard_normal((4, 8, 64)), bits, 64, dtype)
            add(f"hd128_{dtype}_b{bits}", rng.standard_normal((4, 8, 128)), bits, 64, dtype)
            add(f"ragged100_{dtype}_b{bits}", rng.standard_normal(100), bits, 64, dtype)
            add(f"odd7_{dtype}_b{bits}", rng.standard_normal((3, 7)), bits, 64, dtype)
            add(f"gs3_{dtype}_b{bits}", rng.standard_normal((2, 9)), bits, 3, dtype)
            add(f"gs256_{dtype}_b{bits}", rng.standard_normal(8), bits, 256, dtype)
            add(f"single_{dtype}_b{bits}", np.array([1.5]), bits, 64, dtype)
            add(f"zeros_{dtype}_b{bits}", np.zeros(64), bits, 64, dtype)
            add(f"large_{dtype}_b{bits}", np.array([1000.0, -500.0, 750.0, -250.0] * 16), bits, 64, dtype)
            # ties: values that land exactly on .5 after division by the scale
            add(f"ties_{dtype}_b{bits}", np.array([7.0, 0.5, 1.5, -2.5, 3.5, -0.5, 2.5, -7.0]), bits, 8, dtype)
            add(f"mixedzero_{dtype}_b{bits}", np.concatenate([np.zeros(64), rng.standard_normal(64)]), bits, 64, dtype)
        add(f"tiny_{dtype}_b4", np.array([1e-10, -1e-10, 0.0, 1e-10]), 4, 4, dtype)
    return cases


def gen_kv(out):
    mx_mod = None
    ref = _load_ref_module("ref_quantized_kv_cache", "mlx_flash_compress/quantized_kv_cache.py",
                           extra_path=os.path.join(HERE, "_mlx_standin"))
    import mlx.core as mx  # the stand-in, now on sys.path

    mx_mod = mx
    dt_map = {"bf16": mx_mod.bfloat16, "f32": mx_mod.float32, "f16": mx_mod.float16}
    arrays = {}
    names = []
    for name, x, bits, gs, dtype in kv_cases():
        xa = mx_mod.array(x, dt_map[dtype])
        packed, scales, zeros = ref.quantize_tensor(xa, bits=bits, group_size=gs)
        restored = ref.dequantize_tensor(packed, scales, zeros, bits=bits, original_shape=xa.shape, group_size=gs)
        packed, scales, zeros, restored = (np.asarray(a) for a in (packed, scales, zeros, restored))
        # the oracle must reproduce the reference bit for bit
        op, os_, oz = kv_sym.quantize_tensor(x, bits, gs, dtype)
        orr = kv_sym.dequantize_tensor(op, os_, oz, bits, x.shape, gs)
        assert op.dtype == np.uint8 and np.array_equal(op, packed), name
        assert np.array_equal(os_.view(np.uint32), scales.astype(np.float32).view(np.uint32)), name
        assert np.array_equal(orr.view(np.uint32), restored.astype(np.float32).view(np.uint32)), name
        arrays[f"{name}/x"] = x
        arrays[f"{name}/packed"] = packed.astype(np.uint8)
        arrays[f"{name}/scales"] = scales.astype(np.float32)
        arrays[f"{name}/restored"] = restored.astype(np.float32)
        names.append(f"{name}|{bits}|{gs}|{dtype}")
    arrays["__cases__"] = np.array(names)
    np.savez_compressed(os.path.join(out, "kv_sym.npz"), **arrays)
    return len(names)


def gen_mixed(out):
    ref = _load_ref_module("ref_mixed_precision", "mlx_flash_compress/mixed_precision.py")
    rng = np.random.default_rng(7)
    arrays = {}
    for i, (rows, K, gs) in enumerate([(16, 256, 64), (8, 512, 128), (4, 64, 64)]):
        w = round_to(rng.normal(0, 0.02, (rows, K)).astype(np.float32), "bf16")
        wq, s, b = affine.quantize(w, gs, 4, "bf16", rule="minmax")
        p2, s2, b2, meta = ref.requantize_4bit_to_2bit(wq, s, b)
        d2 = ref.dequantize_2bit(p2, s2, b2, K)
        op2, os2, ob2 = mixed.requantize_4bit_to_2bit(wq, s, b, gs)
        od2 = mixed.dequantize_2bit(op2, os2, ob2, K)
        assert np.array_equal(op2, p2), i
        assert np.array_equal(os2.view(np.uint16), s2.view(np.uint16)), i
        assert np.array_equal(ob2.view(np.uint16), b2.view(np.uint16)), i
        assert np.array_equal(od2.view(np.uint32), d2.view(np.uint32)), i
        arrays[f"c{i}/wq"] = wq
        arrays[f"c{i}/scales"] = s
        arrays[f"c{i}/biases"] = b
        arrays[f"c{i}/packed2"] = p2
        arrays[f"c{i}/scales2"] = s2
        arrays[f"c{i}/biases2"] = b2
        arrays[f"c{i}/deq2"] = d2
        arrays[f"c{i}/meta"] = np.array([rows, K, gs])
    np.savez_compressed(os.path.join(out, "mixed2bit.npz"), **arrays)


def gen_affine(out):
    """Keys ``b{bits}_g{gs}/*`` and ``f16/*``, ``f32/*``: the min/max rule;
    ``mlx/b{bits}_g{gs}/*``: MLX's edge rule on the same weights (both rules
    restated in ``oracle/affine.py``; neither needs the reference tree)."""
    rng = np.random.default_rng(0)
    arrays = {}
    for bits in (2, 4, 8):
        for gs in (32, 64, 128):
            w = round_to(rng.normal(0, 0.02, (48, 256)).astype(np.float32), "bf16")
            w[3, :gs] = np.float32(0.015625)  # constant group -> scale 0, exact bias
            w[5, gs:2 * gs] = 0.0
            w[6, :gs] = -np.abs(w[6, :gs])  # all-negative group: the edge is the min
            w[7, :gs] = np.abs(w[7, :gs])  # all-positive group: the edge is the max
            mq, ms, mb = affine.quantize(w, gs, bits, "bf16", rule="mlx")
            arrays[f"mlx/b{bits}_g{gs}/wq"] = mq
            arrays[f"mlx/b{bits}_g{gs}/scales"] = ms
            arrays[f"mlx/b{bits}_g{gs}/biases"] = mb
            arrays[f"mlx/b{bits}_g{gs}/deq"] = affine.dequantize(mq, ms, mb, gs, bits)
            wq, s, b = affine.quantize(w, gs, bits, "bf16", rule="minmax")
            x = round_to(rng.standard_normal((8, 256)).astype(np.float32), "bf16")
            y = affine.quantized_matmul(x, wq, s, b, True, gs, bits)
            key = f"b{bits}_g{gs}"
            arrays[f"{key}/w"] = w
            arrays[f"{key}/wq"] = wq
            arrays[f"{key}/scales"] = s
            arrays[f"{key}/biases"] = b
            arrays[f"{key}/deq"] = affine.dequantize(wq, s, b, gs, bits)
            arrays[f"{key}/x"] = x
            arrays[f"{key}/y"] = y
    for dtype in ("f16", "f32"):
        w = round_to(rng.normal(0, 0.02, (16, 128)).astype(np.float32), dtype)
        wq, s, b = affine.quantize(w, 64, 4, dtype, rule="minmax")
        mq, ms, mb = affine.quantize(w, 64, 4, dtype, rule="mlx")
        arrays[f"mlx/{dtype}/wq"], arrays[f"mlx/{dtype}/scales"], arrays[f"mlx/{dtype}/biases"] = mq, ms, mb
        arrays[f"mlx/{dtype}/deq"] = affine.dequantize(mq, ms, mb, 64, 4, dtype)
        arrays[f"{dtype}/w"] = w
        arrays[f"{dtype}/wq"] = wq
        arrays[f"{dtype}/scales"] = s
        arrays[f"{dtype}/biases"] = b
        arrays[f"{dtype}/deq"] = affine.dequantize(wq, s, b, 64, 4, dtype)
    np.savez_compressed(os.path.join(out, "affine.npz"), **arrays)


def gen_ep(out):
    ref = _load_ref_module("ref_distributed_experts", "mlx_flash_compress/distributed_experts.py")
    rows = []
    for E in (2, 10, 60, 128, 256):
        for W in (1, 2, 3, 4, 7, 8, 100):
            owners = [ref.ExpertShard(rank=0, world_size=W, total_experts=E).owner_of(e) for e in range(E)]
            for r in range(min(W, 8)):
                s = ref.ExpertShard(rank=r, world_size=W, total_experts=E)
                rows.append({"E": E, "W": W, "rank": r, "owned": s.owned_experts, "owners": owners})
    with open(os.path.join(out, "ep_shard.json"), "w") as f:
        json.dump(rows, f)


def gen_dispatch(out):
    # kernels/ops.py imports the MLX-only loader at import time; provide a
    # placeholder so the pure-NumPy moe_dispatch_numpy can be executed as is.
    pkg = types.ModuleType("mlx_flash_compress")
    pkg.__path__ = []
    kpkg = types.ModuleType("mlx_flash_compress.kernels")
    kpkg.__path__ = []
    loader = types.ModuleType("mlx_flash_compress.kernels.loader")
    loader.get_kernel_loader = lambda: None
    sys.modules.setdefault("mlx_flash_compress", pkg)
    sys.modules.setdefault("mlx_flash_compress.kernels", kpkg)
    sys.modules["mlx_flash_compress.kernels.loader"] = loader
    ref = _load_ref_module("ref_kernel_ops", "mlx_flash_compress/kernels/ops.py")
    rng = np.random.default_rng(3)
    arrays = {}
    for i, (E, H, k) in enumerate([(3, 3, 2), (128, 256, 8), (8, 64, 1)]):
        eo = rng.standard_normal((E, H)).astype(np.float32)
        ids = rng.choice(E, size=k, replace=False)
        wts = rng.random(k).astype(np.float32)
        arrays[f"c{i}/outputs"] = eo
        arrays[f"c{i}/ids"] = ids
        arrays[f"c{i}/weights"] = wts
        arrays[f"c{i}/result"] = ref.moe_dispatch_numpy(eo, ids, wts)
    np.savez_compressed(os.path.join(out, "moe_dispatch.npz"), **arrays)


def _softmax_rows(rng, H, Sq, S):
    z = rng.standard_normal((H, Sq, S)).astype(np.float32) * 2.0
    z = np.exp(z - z.max(axis=-1, keepdims=True))
    return (z / z.sum(axis=-1, keepdims=True)).astype(np.float32)


def gen_evict(out):
    sys.path.insert(0, os.path.join(HERE, "_mlx_standin"))
    import mlx.core as mx

    kvc = _load_ref_module("ref_kv_compression", "mlx_flash_compress/kv_compression.py")
    sll = _load_ref_module("ref_streaming_llm", "mlx_flash_compress/streaming_llm.py")
    arrays = {}
    L, H, D = 2, 4, 8
    for scoring in ("h2o", "scissorhands"):
        rng = np.random.default_rng(7 if scoring == "h2o" else 8)
        cfg = kvc.KVCompressionConfig(budget_ratio=0.8, sink_tokens=2, recent_window=6, scoring=scoring)
        cache = kvc.CompressedKVCache(cfg, L, H, D)
        lens = [0] * L
        steps = [40] + [1] * 6 + [7, 1, 1, 1]
        for si, n in enumerate(steps):
            for li in range(L):
                k = rng.standard_normal((H, n, D)).astype(np.float32)
                v = rng.standard_normal((H, n, D)).astype(np.float32)
                S = lens[li] + n
                a = _softmax_rows(rng, H, n, S)
                ko, vo = cache.update(li, mx.array(k), mx.array(v), mx.array(a))
                lens[li] = ko.shape[1]
                key = f"{scoring}/s{si}/l{li}"
                arrays[f"{key}/k"], arrays[f"{key}/v"], arrays[f"{key}/attn"] = k, v, a
                arrays[f"{key}/k_out"] = np.asarray(ko, np.float32)
                arrays[f"{key}/v_out"] = np.asarray(vo, np.float32)
                imp = cache.tracker._importance[li]
                arrays[f"{key}/imp"] = np.asarray(imp, np.float32) if imp is not None else np.zeros(0, np.float32)
                gi = cache.tracker._global_importance
                arrays[f"{key}/gimp"] = np.asarray(gi, np.float32) if gi is not None else np.zeros(0, np.float32)
        arrays[f"{scoring}/steps"] = np.array(steps)
        arrays[f"{scoring}/stats"] = np.array([cache.get_stats()["compression_count"],
                                               cache.get_stats()["total_evicted"]])
    rng = np.random.default_rng(9)
    cache = sll.StreamingLLMCache(sll.StreamingLLMConfig(num_sink_tokens=4, window_size=16), L, H, D)
    steps = [10, 3, 3, 3, 3, 1, 1, 20, 1]
    for si, n in enumerate(steps):
        for li in range(L):
            k = rng.standard_normal((H, n, D)).astype(np.float32)
            v = rng.standard_normal((H, n, D)).astype(np.float32)
            ko, vo = cache.update(li, mx.array(k), mx.array(v))
            key = f"stream/s{si}/l{li}"
            arrays[f"{key}/k"], arrays[f"{key}/v"] = k, v
            arrays[f"{key}/k_out"] = np.asarray(ko, np.float32)
            arrays[f"{key}/v_out"] = np.asarray(vo, np.float32)
            arrays[f"{key}/pos"] = np.asarray(cache.get_positions(li)).astype(np.int32)
    arrays["stream/steps"] = np.array(steps)
    st = cache.get_stats()
    arrays["stream/stats"] = np.array([st["eviction_count"], st["total_evicted_tokens"], st["current_length"]])
    np.savez_compressed(os.path.join(out, "kv_evict.npz"), **arrays)


def main():
    out = HERE
    if "--affine-only" in sys.argv:
        gen_affine(out)
        print("golden vectors written: affine")
        return
    n = gen_kv(out)
    gen_mixed(out)
    gen_affine(out)
    gen_ep(out)
    gen_dispatch(out)
    gen_evict(out)
    print(f"golden vectors written: {n} KV cases + mixed/affine/ep/dispatch/evict")


if __name__ == "__main__":
    main()
