"""The end-to-end gate: synthetic stores made by the reference's own `tlmc`
and the reference's decoder step with its MoE blocks on the GPU.

TEST INFRASTRUCTURE ONLY (imported by tests/ and tests/golden/make_golden.py).
It drives three things built by oracle/Makefile (`make -C oracle gate`):

- `_ref/bin/tlmc`: the reference's compiler, built from its sources. store()
  runs `tlmc synth` + `tlmc compile --profile exact` once per variant into
  `_ref/stores/<name>/` (the packet file is deterministic for a given seed);
- `_ref/libtlmgate.so` / `_ref/libtlmgate_cr.so` (ref_gate.c): the reference's
  tlm_model.c with the store opened as `tierlm` opens it, stepping tokens
  through tlm_model_step (REF), a call-for-call restatement of it (CPU), or
  the restatement with every moe() served by libtlmg's tlmg_moe_layer_ex
  (GPU), or libtlmg's whole decoder step, tlmg_decode_step, with the
  store's attention, embedding and lm_head weights and the KV pages on the
  GPU too (STEP). The `_cr` build binds tlm_model.c's expf to a correctly rounded
  expf, the one the CUDA tier computes.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import shutil
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
TLMC = HERE / "_ref" / "bin" / "tlmc"
STORE_DIR = HERE / "_ref" / "stores"
LIBS = {False: HERE / "_ref" / "libtlmgate.so", True: HERE / "_ref" / "libtlmgate_cr.so"}

REF, CPU, GPU, STEP = 0, 1, 2, 3

_TINY = ["--layers", "4", "--experts", "32", "--top-k", "4", "--shared", "1", "--d-model", "512", "--heads", "8",
         "--kv-heads", "2", "--head-dim", "64", "--vocab", "4096", "--d-expert", "256", "--seed", "1"]
# name -> (tlmc synth arguments, extra tlmc compile arguments)
STORES = {
    # BASELINE config 1 as written: Q6_K experts, Q8_0 dense (tlmc compile defaults)
    "config1": (_TINY, []),
    # the same checkpoint with Q4_K experts
    "config1_q4k": (_TINY, ["--experts", "q4_k"]),
    # a dense-FFN prefix layer (first_k_dense_replace) before the routed layers
    "dense": (["--layers", "3", "--experts", "16", "--top-k", "2", "--shared", "1", "--d-model", "512",
               "--heads", "8", "--kv-heads", "2", "--head-dim", "64", "--vocab", "4096", "--d-expert", "256",
               "--dense-layers", "1", "--dense-ffn", "512", "--seed", "3"], []),
}


def available() -> bool:
    return TLMC.exists() and LIBS[False].exists() and LIBS[True].exists()


def _env() -> dict:
    etc = STORE_DIR / "etc"
    etc.mkdir(parents=True, exist_ok=True)
    return dict(os.environ, TIERLM_ETC=str(etc))   # never read the machine's /etc/tierlm


def store(name: str) -> Path:
    """Manifest path of store `name`, made by tlmc on first use."""
    d = STORE_DIR / name
    man = d / "m.tlmm"
    if man.exists() and (d / "d0" / "m.tlmp").exists():
        return man
    synth, extra = STORES[name]
    if d.exists():
        shutil.rmtree(d)
    d.mkdir(parents=True)
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "src"
        subprocess.run([str(TLMC), "synth", "--out", str(src), *synth], check=True, env=_env(),
                       capture_output=True)
        subprocess.run([str(TLMC), "compile", str(src), "--out", str(man), "--drives", str(d / "d0"),
                        "--profile", "exact", *extra], check=True, env=_env(), capture_output=True)
    shutil.rmtree(d / "m.work", ignore_errors=True)   # compiler scratch (pass-2 store, audit log)
    return man


def store_sha256(name: str) -> str:
    """sha256 of the store's packet file (pins the weights a golden was made on)."""
    h = hashlib.sha256()
    with open(store(name).parent / "d0" / "m.tlmp", "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def xorshift_prompt(n: int, vocab: int, seed: int = 42) -> np.ndarray:
    """cmd_bench's deterministic prompt (reference src/bin/tierlm.c:711-715)."""
    x = seed & 0xFFFFFFFFFFFFFFFF
    out = np.zeros(n, np.int32)
    m = 0xFFFFFFFFFFFFFFFF
    for i in range(n):
        x ^= (x << 13) & m
        x ^= x >> 7
        x ^= (x << 17) & m
        out[i] = x % vocab
    return out


_P, _I = C.c_void_p, C.c_int
_SIGS = {
    "gate_errmsg": (C.c_char_p, []),
    "gate_open": (_P, [C.c_char_p, _I, _I]),
    "gate_close": (None, [_P]),
    "gate_geom": (_I, [_P, _P]),
    "gate_geomf": (_I, [_P, _P]),
    "gate_attach_gpu": (_I, [_P, _I]),
    "gate_reset": (_I, [_P]),
    "gate_hook_enable": (_I, [_P, _I]),
    "gate_hook_read": (_I, [_P, _I, _P, _P, _P]),
    "gate_step": (_I, [_P, _I, _I, _P]),
    "gate_generate": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "gate_teacher": (_I, [_P, _I, _P, _I, _P]),
    "gate_moe": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "gate_layer_tensor": (C.c_int64, [_P, _I, _I, _P, C.POINTER(_I)]),
    "gate_expert": (C.c_int64, [_P, _I, _I, _P, C.POINTER(_I), C.POINTER(C.c_uint32)]),
}
_libs: dict[bool, C.CDLL] = {}


def _lib(cr: bool) -> C.CDLL:
    if cr not in _libs:
        L = C.CDLL(str(LIBS[cr]))
        for n, (res, args) in _SIGS.items():
            f = getattr(L, n)
            f.restype, f.argtypes = res, args
        _libs[cr] = L
    return _libs[cr]


def _ptr(a):
    return None if a is None else a.ctypes.data


class Gate:
    """One opened store: the reference model plus, after attach_gpu(), a
    libtlmg context holding every layer's MoE block on the GPU."""

    def __init__(self, name: str, cr: bool = False, threads: int = 0, max_ctx: int = 256):
        self.L = _lib(cr)
        self.h = self.L.gate_open(str(store(name)).encode(), threads, max_ctx)
        if not self.h:
            raise RuntimeError(self.L.gate_errmsg().decode())
        g = np.zeros(8, np.int32)
        self.L.gate_geom(self.h, _ptr(g))
        (self.n_layers, self.d_model, self.vocab, self.n_experts, self.top_k, self.d_expert, self.d_shared,
         self.n_dense) = (int(v) for v in g)
        gf = np.zeros(3, np.float32)
        self.L.gate_geomf(self.h, _ptr(gf))
        self.router, self.routed_scale, self.norm_eps = int(gf[0]), float(gf[1]), float(gf[2])

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(f"gate error {rc}: {self.L.gate_errmsg().decode()}")

    def attach_gpu(self, device: int = 0) -> None:
        self._check(self.L.gate_attach_gpu(self.h, device))

    def teacher(self, mode: int, seq: np.ndarray) -> np.ndarray:
        """Logits [n][vocab] of every position of a teacher-forced run."""
        seq = np.ascontiguousarray(seq, np.int32)
        out = np.zeros((len(seq), self.vocab), np.float32)
        self._check(self.L.gate_teacher(self.h, mode, _ptr(seq), len(seq), _ptr(out)))
        return out

    def generate(self, mode: int, prompt: np.ndarray, n_gen: int) -> tuple[np.ndarray, np.ndarray]:
        """Greedy tokens [n_gen] after the prompt, and the logits of every step."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        toks = np.zeros(n_gen, np.int32)
        lg = np.zeros((len(prompt) + n_gen - 1, self.vocab), np.float32)
        self._check(self.L.gate_generate(self.h, mode, _ptr(prompt), len(prompt), n_gen, _ptr(toks), _ptr(lg)))
        return toks, lg

    def hook(self, on: bool) -> None:
        self.L.gate_hook_enable(self.h, 1 if on else 0)

    def hook_read(self, layer: int):
        k = max(self.top_k, 1)
        ids, w, on = np.zeros(k, np.int32), np.zeros(k, np.float32), np.zeros(k, np.float32)
        n = self.L.gate_hook_read(self.h, layer, _ptr(ids), _ptr(w), _ptr(on))
        return n, ids, w, on

    def moe(self, mode: int, layer: int, h: np.ndarray):
        """One moe() call (REF: the reference's own; GPU: tlmg) on a copy of h:
        (h_out, ids, w, onorm)."""
        h = np.array(h, np.float32, copy=True)
        k = max(self.top_k, 1)
        ids, w, on = np.full(k, -1, np.int32), np.zeros(k, np.float32), np.zeros(k, np.float32)
        self._check(self.L.gate_moe(self.h, mode, layer, _ptr(h), _ptr(ids), _ptr(w), _ptr(on)))
        return h, ids, w, on

    def layer_tensor(self, layer: int, which: int):
        dt = C.c_int()
        n = self.L.gate_layer_tensor(self.h, layer, which, None, C.byref(dt))
        if n <= 0:
            return None, None
        buf = np.zeros(n, np.uint8)
        self.L.gate_layer_tensor(self.h, layer, which, _ptr(buf), C.byref(dt))
        return buf, dt.value

    def expert(self, layer: int, e: int):
        """(payload uint8, item_off[3], dtype) of one routed expert."""
        dt = C.c_int()
        off = (C.c_uint32 * 3)()
        n = self.L.gate_expert(self.h, layer, e, None, C.byref(dt), off)
        if n <= 0:
            raise RuntimeError(f"expert {layer}:{e}: {self.L.gate_errmsg().decode()}")
        buf = np.zeros(n + 256, np.uint8)
        self.L.gate_expert(self.h, layer, e, _ptr(buf), C.byref(dt), off)
        return buf, tuple(int(v) for v in off), dt.value

    def oracle_layer(self, layer: int):
        """The layer's tensors as oracle.moe_layer arguments: (layer dict, experts)."""
        norm, _ = self.layer_tensor(layer, 0)
        lay = {"ffn_norm": norm.view(np.float32)}
        dense = [self.layer_tensor(layer, w) for w in (7, 8, 9)]
        if dense[0][0] is not None:
            d_ffn = dense[0][0].size // _row_bytes(dense[0][1], self.d_model)
            lay["dense"] = (tuple(d[1] for d in dense), [d[0] for d in dense], d_ffn)
            return lay, []
        rw, rdt = self.layer_tensor(layer, 1)
        lay.update(router_w=rw, router_dt=rdt, router_rb=_row_bytes(rdt, self.d_model))
        bias, _ = self.layer_tensor(layer, 2)
        if bias is not None:
            lay["router_bias"] = bias.view(np.float32)
        sh = [self.layer_tensor(layer, w) for w in (3, 4, 5)]
        if sh[0][0] is not None:
            lay["shared"] = (tuple(s[1] for s in sh), [s[0] for s in sh])
            gi, _ = self.layer_tensor(layer, 6)
            if gi is not None:
                lay["shared_gate_inp"] = gi.view(np.float32)
        experts = []
        for e in range(self.n_experts):
            buf, off, dt = self.expert(layer, e)
            experts.append((buf, off, (dt, dt, dt)))
        return lay, experts

    def geom(self) -> dict:
        return dict(d_model=self.d_model, d_expert=self.d_expert, d_shared=self.d_shared, n_experts=self.n_experts,
                    top_k=self.top_k, router=self.router, routed_scale=self.routed_scale, norm_eps=self.norm_eps)

    def close(self) -> None:
        if self.h:
            self.L.gate_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def _row_bytes(dt: int, n: int) -> int:
    import oracle
    return oracle.row_bytes(dt, n)
