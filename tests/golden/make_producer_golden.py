"""Record the reference's producer outputs as golden fixtures (run on a B200).

    python tests/golden/make_producer_golden.py [--out tests/golden/producers_ref.json]

Runs the reference's own ``nvfp4_norm_pack.cu`` and ``nvfp4_attention_front.cu``
(compiled for sm_100a from its sources by ``oracle/build_ref.py``) and the
restatement of its FP8 gate epilogue (``oracle/gpu_checks.cu``) on seeded
inputs that numpy regenerates anywhere, and writes per case:

* the SHA-256 of every output tensor of the reference kernel;
* the CUDA ``rsqrtf`` / ``expf`` values the CPU oracle needs for these inputs
  wherever they differ from the correctly rounded host values (fp32 input
  bits -> output bits), so the CPU tests can rebuild the outputs exactly with
  :class:`oracle.producers.RecordedMath`.

The CPU test ``tests/test_oracle_pins.py::test_oracle_reproduces_reference_producer_bytes``
regenerates the inputs with :func:`case_inputs`, runs the oracle and compares
the hashes.  Only this script needs a GPU and the reference build.
"""

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from oracle import formats as F  # noqa: E402
from oracle import model as OM  # noqa: E402
from oracle import producers as P  # noqa: E402

CASES = {
    "norm_pack": [dict(rows=64, seed=1, std=1.0, g=672.0), dict(rows=33, seed=2, std=40.0, g=16.8)],
    "attention_front": [dict(rows=64, qheads=4, kvheads=2, page_size=32, seed=3, history=700),
                        dict(rows=40, qheads=2, kvheads=1, page_size=32, seed=4, history=0)],
    "gate_static": [dict(rows=64, cols=1024, seed=5, scale=0.0123)],
}
KG, VG = np.float32(16 / 2688), np.float32(8 / 2688)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16(rng, shape, std=1.0):
    return F.bf16_round((rng.standard_normal(shape) * std).astype(np.float32))


def case_inputs(kind, spec):
    """Seeded inputs of one case as numpy arrays (bf16 values held in fp32)."""
    rng = np.random.default_rng(spec["seed"])
    if kind == "norm_pack":
        rows = spec["rows"]
        return dict(x=bf16(rng, (rows, 5120), spec["std"]), r=bf16(rng, (rows, 5120), spec["std"]),
                    w=bf16(rng, (5120,), 0.05))
    if kind == "attention_front":
        rows, qh, kvh, ps, hist = (spec[k] for k in ("rows", "qheads", "kvheads", "page_size", "history"))
        qkv = bf16(rng, (rows, (2 * qh + 2 * kvh) * 256), 1.5)
        qw, kw = bf16(rng, (256,), 0.05), bf16(rng, (256,), 0.05)
        maxpos = hist + rows
        pages = (maxpos + ps - 1) // ps + 2
        table = rng.permutation(pages)[: (maxpos + ps - 1) // ps]
        pos = np.arange(hist, hist + rows, dtype=np.int64)
        slots = (table[pos // ps] * ps + pos % ps).astype(np.int64)
        slots[rng.random(rows) < 0.1] = -1
        return dict(qkv=qkv, qw=qw, kw=kw, cos=OM.rope_table(maxpos + 3, 256, 1e6), pos=pos, slots=slots,
                    pages=pages)
    if kind == "gate_static":
        return dict(values=bf16(rng, (spec["rows"], spec["cols"]), 3.0),
                    gates=bf16(rng, (spec["rows"], spec["cols"]), 2.0))
    raise KeyError(kind)


def oracle_outputs(kind, spec):
    """The CPU oracle's outputs of one case (uses the current P.MATH)."""
    a = case_inputs(kind, spec)
    if kind == "norm_pack":
        q, sf, upd = P.norm_pack(a["x"], a["r"], a["w"], np.float32(spec["g"]))
        return dict(q=q, scales=sf, updated=F.bf16_bits(upd))
    if kind == "attention_front":
        qh, kvh, ps = spec["qheads"], spec["kvheads"], spec["page_size"]
        kv = OM.KVCache(OM.Shape(1, qh * 256, qh, kvh, 256, 1024, page_size=ps), a["pages"])
        q, gate = P.qk_rope_append(a["qkv"], a["pos"], a["qw"], a["kw"], a["cos"], a["slots"], KG, VG, kv.k, kv.v,
                                   kv.ks, kv.vs, qheads=qh, kvheads=kvh, head_dim=256, page_size=ps)
        return dict(q=F.bf16_bits(q), gate=F.bf16_bits(gate), k=kv.k, v=kv.v, ks=kv.ks, vs=kv.vs)
    if kind == "gate_static":
        codes, _ = P.gate_fp8(a["values"], a["gates"], static_scale=np.float32(spec["scale"]))
        return dict(fp8=codes)
    raise KeyError(kind)


class _Recorder(P.HostMath):
    """CUDA's values, remembering where they differ from the host ones."""

    def __init__(self, cuda):
        self.cuda = cuda
        self.diff = {"rsqrt": {}, "exp": {}}

    def _rec(self, which, x, got):
        host = getattr(P.HostMath, which)(self, x)
        xb = np.asarray(x, dtype=np.float32).reshape(-1).view(np.uint32)
        gb, hb = got.reshape(-1).view(np.uint32), host.reshape(-1).view(np.uint32)
        for i in np.nonzero(gb != hb)[0]:
            self.diff[which][int(xb[i])] = int(gb[i])
        return got

    def rsqrt(self, x):
        return self._rec("rsqrt", x, self.cuda.rsqrt(x))

    def exp(self, x):
        return self._rec("exp", x, self.cuda.exp(x))


def reference_outputs(kind, spec):
    """Outputs of the reference kernels (GPU) for one case."""
    import torch

    import __graft_entry__

    __graft_entry__.load_package()
    sys.path.insert(0, str(REPO / "tests"))
    import test_ref_pin_gpu as T
    from oracle import cuda_math

    dev = torch.device("cuda:0")
    a = case_inputs(kind, spec)

    def to_bf16(x):
        return torch.from_numpy(x).to(torch.bfloat16).to(dev)

    def bits(t):
        return t.view(torch.int16).cpu().numpy().view(np.uint16)

    if kind == "norm_pack":
        lib = T.ct.CDLL(str(T.REF / "libref_norm_pack.so"))
        q, sc, upd = T.run_norm_pack(lib, to_bf16(a["x"]), to_bf16(a["r"]), to_bf16(a["w"]),
                                     torch.tensor([spec["g"]], dtype=torch.float32, device=dev), spec["rows"])
        return dict(q=q.cpu().numpy(), scales=sc.cpu().numpy(), updated=bits(upd))
    if kind == "attention_front":
        lib = T.ct.CDLL(str(T.REF / "libref_attention_front.so"))
        args = dict(qkv=to_bf16(a["qkv"]), qw=to_bf16(a["qw"]), kw=to_bf16(a["kw"]),
                    cos=torch.from_numpy(a["cos"]).to(dev), pos=torch.from_numpy(a["pos"]).to(dev),
                    slots=torch.from_numpy(a["slots"]).to(dev), pages=a["pages"], page_size=spec["page_size"],
                    rows=spec["rows"], qh=spec["qheads"], kvh=spec["kvheads"],
                    kg=torch.tensor([KG], device=dev), vg=torch.tensor([VG], device=dev), slot_rows=spec["rows"])
        out = T.run_front(lib, args)
        res = {k: v.cpu().numpy() for k, v in out.items() if k not in ("q", "gate")}
        res["q"], res["gate"] = bits(out["q"]), bits(out["gate"])
        return res
    if kind == "gate_static":
        codes = cuda_math.gate_fp8_static_reference(to_bf16(a["values"]), to_bf16(a["gates"]),
                                                    torch.tensor([spec["scale"]], dtype=torch.float32,
                                                                 device=dev))
        return dict(fp8=codes.cpu().numpy())
    raise KeyError(kind)


def main():
    from oracle import cuda_math

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "producers_ref.json"))
    out_path = Path(ap.parse_args().out)
    result = dict(generator="tests/golden/make_producer_golden.py", cases={})
    for kind, specs in CASES.items():
        for spec in specs:
            ref = reference_outputs(kind, spec)
            rec = _Recorder(cuda_math.CudaMath())
            with P.use_math(rec):
                ours = oracle_outputs(kind, spec)
            agree = {k: bool(np.array_equal(np.asarray(ours[k]).reshape(-1), np.asarray(ref[k]).reshape(-1)))
                     for k in ref}
            result["cases"].setdefault(kind, []).append(dict(
                spec=spec, sha256={k: sha(v) for k, v in ref.items()}, oracle_agrees=agree,
                rsqrt_differs={str(k): v for k, v in sorted(rec.diff["rsqrt"].items())},
                exp_differs={str(k): v for k, v in sorted(rec.diff["exp"].items())}))
            print(kind, spec, agree, {k: len(v) for k, v in rec.diff.items()}, flush=True)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(json.dumps(result, indent=1) + "\n")
    print("wrote", out_path)


if __name__ == "__main__":
    main()
