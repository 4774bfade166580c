"""CPU restatement of ltx-weights' WeightStore / LoraFile / KeyMap.

TEST INFRASTRUCTURE ONLY.  This module checks the CUDA library; it is never
imported by the product path (ltx-rust_b200/).  Only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline leg use it.

Follows, line by line:
  - WeightStore::open       crates/ltx-weights/src/store.rs:124-208
    (key renaming, duplicate-key rejection, FP8 `_scale` sibling hiding :174-187)
  - WeightStore::read       store.rs:479-521  (decode, fma(scale, v, 0), deltas)
  - WeightStore::merge_lora store.rs:542-640  (pairing, rank/shape checks,
                                               alpha default, coefficient :615)
  - LowRankDelta::add_to    store.rs:767-793  (the bit-exact FMA chain)
  - LoraFile                crates/ltx-weights/src/lora.rs:43-209
  - KeyMap identity/transformer  crates/ltx-weights/src/key_map.rs:90-111, 237-273
The numeric core (decode + scale + FMA chain + bf16 rounding) is the C file
oracle/fp8_merge.c, so the bit pattern is decided by IEEE fmaf, not by numpy.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle_fp8.so")

DTYPE_CODE = {"F32": 0, "F16": 1, "BF16": 2, "F8_E4M3": 3, "F8_E5M2": 4}
DTYPE_SIZE = {"F32": 4, "F16": 2, "BF16": 2, "F8_E4M3": 1, "F8_E5M2": 1,
              "F64": 8, "I64": 8, "U64": 8, "I32": 4, "U32": 4, "I16": 2, "U16": 2,
              "I8": 1, "U8": 1, "BOOL": 1}

_lib = None


def lib() -> ctypes.CDLL:
    """Load (building on first use) the C oracle."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            import subprocess
            subprocess.run(["make", "-C", _HERE], check=True, capture_output=True)
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_read_weight.restype = ctypes.c_int
        L.oracle_read_weight.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
            ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float),
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.oracle_lora_coeff.restype = ctypes.c_float
        L.oracle_lora_coeff.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int]
        for name in ("oracle_decode_e4m3fn", "oracle_decode_e5m2"):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [ctypes.c_uint8]
        for name in ("oracle_fmaf",):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [ctypes.c_float] * 3
        L.oracle_expf.restype = ctypes.c_float
        L.oracle_crossfade_blend.restype = None
        L.oracle_crossfade_blend.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_longlong,
                                             ctypes.c_void_p]
        L.oracle_expf.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


class WeightError(Exception):
    """Mirror of WeightError (crates/ltx-weights/src/error.rs:7-101); `kind` names the variant."""

    def __init__(self, kind: str, msg: str = ""):
        super().__init__(f"{kind}: {msg}")
        self.kind = kind


# ── safetensors container ─────────────────────────────────────────────────────

def read_safetensors(path: str):
    """Return (metadata: dict[str,str], tensors: dict[name -> (dtype, shape, bytes)])."""
    with open(path, "rb") as f:
        data = f.read()
    (hlen,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + hlen])
    meta = header.pop("__metadata__", None) or {}
    base = 8 + hlen
    tensors = {}
    for name, info in header.items():
        s, e = info["data_offsets"]
        tensors[name] = (info["dtype"], list(info["shape"]), data[base + s: base + e])
    return meta, tensors


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None):
    """tensors: name -> (dtype_str, shape, raw_bytes)."""
    header = {}
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    off = 0
    parts = []
    for name, (dt, shape, raw) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        parts.append(raw)
        off += len(raw)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for p in parts:
            f.write(p)


def decode_to_f32(dtype: str, raw: bytes) -> np.ndarray:
    """decode_to_f32 (store.rs:672-729) / decode_lora_bytes (lora.rs:176-209)."""
    if dtype == "F32":
        return np.frombuffer(raw, dtype="<f4").astype(np.float32)
    if dtype == "F16":
        return np.frombuffer(raw, dtype="<f2").astype(np.float32)
    if dtype == "BF16":
        u = np.frombuffer(raw, dtype="<u2").astype(np.uint32) << 16
        return u.view(np.float32)
    if dtype in ("F8_E4M3", "F8_E5M2"):
        fn = lib().oracle_decode_e4m3fn if dtype == "F8_E4M3" else lib().oracle_decode_e5m2
        lut = np.array([fn(b) for b in range(256)], dtype=np.float32)
        return lut[np.frombuffer(raw, dtype=np.uint8)]
    raise WeightError("UnsupportedDtype", dtype)


# ── KeyMap ────────────────────────────────────────────────────────────────────

class KeyMap:
    """key_map.rs:90-111 (identity, transformer) and apply_key :237-273."""

    def __init__(self, rules):
        self.rules = rules

    @staticmethod
    def identity():
        return KeyMap([])

    @staticmethod
    def transformer():
        return KeyMap([("require", ["model.diffusion_model."]),
                       ("replace", "model.diffusion_model.", "")])

    def apply_key(self, key: str):
        for rule in self.rules:
            if rule[0] == "require":
                if rule[1] and not any(key.startswith(p) for p in rule[1]):
                    return None
            elif rule[0] == "replace":
                key = key.replace(rule[1], rule[2])
        return key


# ── LoRA ─────────────────────────────────────────────────────────────────────

class LoraFile:
    """lora.rs:43-153."""

    def __init__(self, path: str):
        self.metadata, self.tensors = read_safetensors(path)

    def read_f32(self, name):
        if name not in self.tensors:
            return None
        dt, shape, raw = self.tensors[name]
        try:
            return shape, decode_to_f32(dt, raw)
        except WeightError as e:
            raise WeightError("UnsupportedDtype", name) from e

    def ic_layout(self):
        """lora.rs:105-110: (reference_downscale_factor, reference_temporal_scale_factor), default 1."""
        def u32(k):
            v = self.metadata.get(k)
            try:
                return int(v.strip()) if v is not None else None
            except ValueError:
                return None
        d = u32("reference_downscale_factor") or 1
        t = u32("reference_temporal_scale_factor") or 1
        return d, t


@dataclass
class LowRankDelta:
    """store.rs:756-763."""
    b: np.ndarray          # [out, rank] f32
    a: np.ndarray          # [rank, in] f32
    out_features: int
    rank: int
    in_features: int
    scale: float


@dataclass
class MergeReport:
    matched_keys: list = field(default_factory=list)
    unmatched_lora_keys: list = field(default_factory=list)


# ── WeightStore ──────────────────────────────────────────────────────────────

class WeightStore:
    def __init__(self, paths, keymap: KeyMap):
        self.entries = {}
        self.metadata = {}
        for p in paths:
            meta, tensors = read_safetensors(p)
            for k, v in meta.items():
                self.metadata.setdefault(k, v)
            for name, ent in tensors.items():
                renamed = keymap.apply_key(name)
                if renamed is None:
                    continue
                if renamed in self.entries:
                    raise WeightError("DuplicateKey", renamed)
                self.entries[renamed] = ent
        # store.rs:174-187: FP8 scale siblings are internal
        self.scale_keys = {k for k in self.entries
                           if k.endswith("_scale") and k[:-6] in self.entries
                           and self.entries[k[:-6]][0] in ("F8_E4M3", "F8_E5M2")}
        self.lora_deltas: dict[str, list[LowRankDelta]] = {}

    def keys(self):
        return [k for k in self.entries if k not in self.scale_keys]

    def contains(self, key):
        return key in self.entries and key not in self.scale_keys

    def shape(self, key):
        if key not in self.entries:
            raise WeightError("MissingKey", key)
        return self.entries[key][1]

    def config(self):
        if "config" not in self.metadata:
            raise WeightError("MissingConfig")
        return json.loads(self.metadata["config"])

    def scale_of(self, key):
        """(has_scale, scale) as read() applies it (store.rs:498-508, decode_scalar_f32 :732-735)."""
        dt = self.entries[key][0]
        sk = key + "_scale"
        if dt in ("F8_E4M3", "F8_E5M2") and sk in self.entries:
            sdt, _, sraw = self.entries[sk]
            v = decode_to_f32(sdt, sraw)
            return True, float(v[0]) if v.size else 1.0
        return False, 1.0

    def read(self, key, want="f32", n_threads=1):
        """WeightStore::read; want = "f32" | "bf16" (bf16 = RNE of the f32 result)."""
        if key not in self.entries:
            raise WeightError("MissingKey", key)
        dt, shape, raw = self.entries[key]
        if dt not in DTYPE_CODE:
            raise WeightError("UnsupportedDtype", key)
        n = int(np.prod(shape)) if shape else 1
        if len(raw) != n * DTYPE_SIZE[dt]:
            raise WeightError("InvalidTensorData", key)
        has_scale, scale = self.scale_of(key)
        deltas = self.lora_deltas.get(key, [])
        if deltas:
            out, inn = deltas[0].out_features, deltas[0].in_features
        else:
            inn = shape[-1] if shape else 1
            out = n // inn if inn else 0
        return read_raw(raw, dt, has_scale, scale, out, inn, deltas, want, n_threads).reshape(shape)

    def merge_lora(self, lora: LoraFile, strength: float) -> MergeReport:
        report = MergeReport()
        suffix = ".lora_A.weight"
        pending = []
        for key_a in [k for k in lora.tensors if k.endswith(suffix)]:
            prefix = key_a[: -len(suffix)]
            base_key, key_b = prefix + ".weight", prefix + ".lora_B.weight"
            if base_key not in self.entries:
                report.unmatched_lora_keys.append(key_a)
                continue
            ra = lora.read_f32(key_a)
            if ra is None:
                report.unmatched_lora_keys.append(key_a)
                continue
            rb = lora.read_f32(key_b)
            if rb is None:
                report.unmatched_lora_keys.append(key_a)
                continue
            (shape_a, a), (shape_b, b) = ra, rb
            rank_a = shape_a[0] if shape_a else 0
            rank_b = shape_b[1] if len(shape_b) > 1 else 0
            if rank_a != rank_b or rank_a == 0:
                raise WeightError("LoraRankMismatch", base_key)
            es = self.entries[base_key][1]
            out_f = es[0] if es else 0
            in_f = es[1] if len(es) > 1 else 1
            b_out = shape_b[0] if shape_b else 0
            a_in = shape_a[1] if len(shape_a) > 1 else 0
            if b_out != out_f or a_in != in_f:
                raise WeightError("LoraShapeMismatch", base_key)
            alpha_r = lora.read_f32(prefix + ".alpha")
            alpha = float(alpha_r[1][0]) if alpha_r is not None and alpha_r[1].size else float(np.float32(rank_a))
            coeff = lib().oracle_lora_coeff(strength, alpha, rank_a)
            pending.append((base_key, LowRankDelta(np.ascontiguousarray(b, np.float32),
                                                   np.ascontiguousarray(a, np.float32),
                                                   out_f, rank_a, in_f, coeff)))
            report.matched_keys.append(base_key)
        if not report.matched_keys and report.unmatched_lora_keys:
            raise WeightError("NoLoraMatches")
        for k, d in pending:
            self.lora_deltas.setdefault(k, []).append(d)
        return report


def read_raw(raw: bytes, dt: str, has_scale: bool, scale: float, out: int, inn: int,
             deltas, want="f32", n_threads=1) -> np.ndarray:
    """One weight read through the C core; returns f32 or uint16 (bf16 bits)."""
    L = lib()
    nd = len(deltas)
    for d in deltas:
        if d.out_features != out or d.in_features != inn:
            raise WeightError("LoraShapeMismatch", "")
    base = np.frombuffer(raw, dtype=np.uint8)
    A = (ctypes.c_void_p * max(nd, 1))(*[d.a.ctypes.data for d in deltas])
    B = (ctypes.c_void_p * max(nd, 1))(*[d.b.ctypes.data for d in deltas])
    R = (ctypes.c_int * max(nd, 1))(*[d.rank for d in deltas])
    C = (ctypes.c_float * max(nd, 1))(*[d.scale for d in deltas])
    dst = np.empty(out * inn, dtype=np.float32 if want == "f32" else np.uint16)
    rc = L.oracle_read_weight(base.ctypes.data, DTYPE_CODE[dt], int(has_scale), scale, out, inn, nd,
                              A, B, R, C,
                              dst.ctypes.data if want == "f32" else None,
                              dst.ctypes.data if want != "f32" else None, n_threads)
    if rc != 0:
        raise WeightError("UnsupportedDtype", dt)
    return dst


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Vectorised RNE f32 -> bf16 bits, same rule as oracle_f32_to_bf16 (half 2.7.1)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rnd = ((u & 0x8000) != 0) & ((u & (3 * 0x8000 - 1)) != 0)
    r = (u >> 16) + rnd.astype(np.uint32)
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)
