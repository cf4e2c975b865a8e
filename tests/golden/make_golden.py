"""Generate the golden fixtures in this directory from the REFERENCE's own Python code.

Runs only where davetha/r9700-lru-expert-cache is checked out (pass its path as argv[1]);
the fixtures it writes are committed so the tests never need the reference at run time.

What runs from the reference, unmodified:
* ``kernels/draft_w4_lmhead.py`` -- ``quantize_w4``, ``pack_w4a16``, ``unpack_w4``, the
  launch-config helpers ``_legal``/``pick_cfg``. Loaded with a stub for the fork-only
  ``vllm.model_executor.kernels.r4d_lib`` (``available() -> False``).
* ``kernels/fp8_target_lmhead.py`` -- ``pack_fp8_block``, with an identity stub for the
  gfx1201-only ``shuffle_weight_gfx1201`` so the weight comes out row-major.
* ``tests/lru/test_lru.py`` -- ``ref_step``, the reference's independent numpy model of
  ``lru_manage_k``, extracted from the file's AST (the module itself dlopens the HIP
  library at import, so it cannot be imported here).
* ``tests/lru/test_victim_equiv.py`` -- its ``Case`` class (state construction of the 19
  victim-selection cases), imported with its device set to CPU.

The routing generators of test_lru.py's suites live inside its ``main()``; they are
restated in ``oracle/lru_oracle.py`` (``suite_gen``) and used here.
"""
from __future__ import annotations

import ast
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import lru_oracle as LO  # noqa: E402


def _stub(name: str, **attrs):
    mod = types.ModuleType(name)
    mod.__dict__.update(attrs)
    sys.modules[name] = mod
    return mod


def load_reference(ref: str):
    _stub("vllm.model_executor.kernels.r4d_lib", available=lambda: False,
          lib=lambda: None)

    class _Fp8HipKernel:
        @staticmethod
        def is_supported():
            return False, "stub"

    _stub("vllm.model_executor.kernels.linear.scaled_mm.fp8hip",
          shuffle_weight_gfx1201=lambda w: w, Fp8HipBlockScaledMMKernel=_Fp8HipKernel)

    def load(path, name):
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    w4 = load(os.path.join(ref, "kernels/draft_w4_lmhead.py"), "_ref_draft_w4_lmhead")
    fp8 = load(os.path.join(ref, "kernels/fp8_target_lmhead.py"), "_ref_fp8_target_lmhead")

    src = open(os.path.join(ref, "tests/lru/test_lru.py")).read()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "ref_step")
    ns = {"np": np}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "test_lru.py", "exec"), ns)

    sys.path.insert(0, os.path.join(ref, "tests/lru"))
    ve = load(os.path.join(ref, "tests/lru/test_victim_equiv.py"), "_ref_victim_equiv")
    ve.DEV = "cpu"
    return w4, fp8, ns["ref_step"], ve


class RefState:
    """The attributes ``ref_step`` reads and writes (tests/lru/test_lru.py:53-72)."""

    def __init__(self, st: LO.LruState):
        self.E, self.S = st.E, st.S
        self.r_table = st.table.copy()
        self.r_cold = st.map_cold.copy()
        self.r_se = st.slot_expert.copy()
        self.r_st = st.slot_stamp.copy()
        self.r_step = int(st.step)

    def digest(self, out) -> int:
        s = LO.LruState(self.r_table, self.r_cold, self.r_se, self.r_st, self.r_step)
        s.n_miss = len(out)
        s.miss = np.array(out, dtype=np.int32).reshape(-1, 2) if out else np.zeros((0, 2), np.int32)
        return LO.state_digest(s)


def gen_w4(w4, out):
    cases = {}
    g = torch.Generator().manual_seed(0)
    shapes = [(48, 256), (200, 256), (32, 384)]
    for i, (n, k) in enumerate(shapes):
        w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
        if i == 2:
            w[0, :128] = 0.0                       # all-zero group -> scale 0
            w[1, :128] = 0.0125                    # constant non-zero group -> code 8
            w[2, 128:256] = w[2, 128:256].abs() + 0.01   # all-positive group -> negative zero
            w[3, 256:384] = -(w[3, 256:384].abs() + 0.01)
        for clip, tag in ((None, "clip"), ((1.0,), "minmax")):
            q, s, z = w4.quantize_w4(w.float(), 128, clip)
            cases[f"{n}x{k}_{tag}_w"] = w.view(torch.int16).numpy()
            cases[f"{n}x{k}_{tag}_q"] = q.numpy()
            cases[f"{n}x{k}_{tag}_scale"] = s.view(torch.int16).numpy()
            cases[f"{n}x{k}_{tag}_zero"] = z.numpy()
            p = w4.pack_w4a16(w, 128, clip_grid=clip)
            cases[f"{n}x{k}_{tag}_wsz"] = p.wsz.numpy()
            up = w4.unpack_w4(p, torch.float32)
            if n == 48:
                cases[f"{n}x{k}_{tag}_unpack"] = up.numpy()
            cases[f"{n}x{k}_{tag}_unpack_sum"] = np.array([up.double().sum().item(),
                                                           up.double().abs().sum().item()])
            cases[f"{n}x{k}_{tag}_npad"] = np.array([p.n_pad])
    # launch-config helpers: every (m, n_pad, k) the tests use
    cfg = []
    for m in (1, 2, 4, 5, 8, 9, 16, 17, 20, 32, 33, 64, 65):
        for n_pad, k in ((151936, 2560), (1008, 256), (1024, 2560), (48, 128)):
            cfg.append([m, n_pad, k, *w4.pick_cfg(m, n_pad, k)])
    cases["pick_cfg"] = np.array(cfg, dtype=np.int64)
    legal = []
    for k in (128, 256, 2560, 1280):
        for wv in (1, 2, 4, 8, 16, 40):
            for sk in (1, 2, 4, 5, 10, 20):
                for npw in (1, 2, 4):
                    for nt in (1, 100):
                        legal.append([k, nt, wv, sk, npw, int(w4._legal(k, nt, wv, sk, npw))])
    cases["legal"] = np.array(legal, dtype=np.int64)
    np.savez_compressed(out, **cases)


def gen_fp8(fp8, out):
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(256, 384, generator=g) * 0.02).bfloat16()
    w[128:256, 128:256] = 0.0                      # all-zero block -> amax floor 1e-12
    w[0, 0] = 3.0                                  # an outlier block
    wq, ws = fp8.pack_fp8_block(w)
    np.savez_compressed(out, w=w.view(torch.int16).numpy(),
                        wq=wq.view(torch.uint8).numpy(), ws=ws.numpy())


def gen_lru(ref_step, ve, out):
    data = {}
    for name, (E, S, nsteps, md, maxi) in LO.SUITES.items():
        rng, st = LO.suite_start(name, seed=0)
        data[f"{name}/init_table"] = st.table.copy()
        data[f"{name}/init_se"] = st.slot_expert.copy()
        rs = RefState(st)
        gen = LO.suite_gen(name)
        ids_all, digests, misses, nmiss = [], [], [], []
        for n in range(nsteps):
            ids = np.asarray(gen(rng, n)).ravel()
            outp = ref_step(rs, ids, md, maxi)
            ids_all.append(ids.astype(np.int32))
            digests.append(rs.digest(outp))
            nmiss.append(len(outp))
            misses.extend([x for pair in outp for x in pair])
        data[f"{name}/ids"] = np.stack(ids_all)
        data[f"{name}/digest"] = np.array(digests, dtype=np.int64)
        data[f"{name}/n_miss"] = np.array(nmiss, dtype=np.int32)
        data[f"{name}/miss"] = np.array(misses, dtype=np.int32)
        data[f"{name}/final_table"] = rs.r_table.copy()
        data[f"{name}/final_se"] = rs.r_se.copy()
        data[f"{name}/final_st"] = rs.r_st.copy()

    cases = [
        ("prod B=1", dict(E=512, S=257, mk=50, k_cold=2, maxi=64, seed=1)),
        ("prod B=4", dict(E=512, S=257, mk=200, k_cold=13, maxi=64, seed=2)),
        ("at the cliff", dict(E=512, S=257, mk=50, k_cold=14, maxi=64, seed=3)),
        ("past the cliff", dict(E=512, S=257, mk=120, k_cold=40, maxi=64, seed=4)),
        ("zero misses", dict(E=512, S=257, mk=50, k_cold=0, maxi=64, seed=5)),
        ("serial n=4", dict(E=512, S=257, mk=50, k_cold=4, maxi=64, seed=18)),
        ("rank n=5", dict(E=512, S=257, mk=50, k_cold=5, maxi=64, seed=19)),
        ("serial, ev=0", dict(E=512, S=24, mk=60, k_cold=3, maxi=64, seed=20)),
        ("serial, ev=2", dict(E=512, S=26, mk=60, k_cold=4, maxi=64, seed=21)),
        ("capped by maxi", dict(E=512, S=257, mk=300, k_cold=200, maxi=8, seed=6)),
        ("tiny maxi", dict(E=512, S=257, mk=100, k_cold=60, maxi=3, seed=15)),
        ("empty slots", dict(E=512, S=257, mk=50, k_cold=10, maxi=64, seed=7, empty=100)),
        ("stamp ties", dict(E=512, S=257, mk=50, k_cold=12, maxi=64, seed=8, tie=True)),
        ("tiny cache", dict(E=512, S=16, mk=50, k_cold=30, maxi=64, seed=9)),
        ("evict-all", dict(E=512, S=24, mk=60, k_cold=50, maxi=64, seed=16)),
        ("evict exhausted", dict(E=512, S=40, mk=200, k_cold=60, maxi=64, seed=10)),
        ("S=1024", dict(E=1024, S=1024, mk=400, k_cold=100, maxi=64, seed=11, resident=600)),
        ("maxi=1024", dict(E=1024, S=1024, mk=900, k_cold=500, maxi=1024, seed=17,
                           resident=400)),
        ("maxi=1", dict(E=512, S=257, mk=50, k_cold=20, maxi=1, seed=12)),
    ]
    names = []
    for i, (name, kw) in enumerate(cases):
        c = ve.Case(**kw)
        p = {k: v.numpy().copy() for k, v in c.pristine.items()}
        key = f"case{i}"
        names.append(name)
        for f in ("table", "map_cold", "slot_expert", "slot_stamp", "step"):
            data[f"{key}/{f}"] = p[f]
        data[f"{key}/ids"] = c.ids.numpy().copy()
        data[f"{key}/params"] = np.array([c.E, c.S, c.mk, c.maxi, c.md], dtype=np.int64)
        st = LO.LruState(p["table"], p["map_cold"], p["slot_expert"], p["slot_stamp"],
                         int(p["step"][0]))
        rs = RefState(st)
        outp = ref_step(rs, c.ids.numpy(), c.md, c.maxi)
        data[f"{key}/digest"] = np.array([rs.digest(outp)], dtype=np.int64)
        data[f"{key}/miss"] = np.array(outp, dtype=np.int32).reshape(-1, 2)
    data["case_names"] = np.array(names)
    np.savez_compressed(out, **data)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("R9700_REF", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py <path to davetha/r9700-lru-expert-cache>")
    w4, fp8, ref_step, ve = load_reference(ref)
    gen_w4(w4, os.path.join(HERE, "w4_reference.npz"))
    gen_fp8(fp8, os.path.join(HERE, "fp8_pack_reference.npz"))
    gen_lru(ref_step, ve, os.path.join(HERE, "lru_reference.npz"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
