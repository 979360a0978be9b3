"""ctypes front-end to the checkers (test infrastructure only).

* ``Oracle``  — liboracle.so, the C restatement in s3t_oracle.c.
* ``Reference`` — oracle/_ref/libsam3ref_v{3,4}.so, the reference's own ggml
  CPU code compiled from its sources by oracle/Makefile (present when it was
  built; it travels with the tree).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module.
"""

from __future__ import annotations

import ctypes as C
import json
import os
import re
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F32, F16, Q8_0 = 0, 1, 8
PREFIX = "backbone.vision_backbone.trunk"

_p = C.c_void_p
_i64 = C.c_int64


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Oracle:
    def __init__(self, path: str | os.PathLike | None = None):
        path = Path(path) if path else HERE / "liboracle.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.lib = L = C.CDLL(str(path))
        L.or_fp32_to_fp16_row.argtypes = [_p, _p, _i64]
        L.or_dequantize.argtypes = [C.c_int, _p, _i64, _p]
        L.or_quantize_q8_0_act.argtypes = [_p, _i64, _p]
        L.or_round_activations.argtypes = [C.c_int, _p, _i64, _p]
        L.or_linear.argtypes = [C.c_int, _p, _i64, _i64, _p, _i64, _p, _p]
        L.or_layer_norm.argtypes = [_p, _i64, _i64, _p, _p, C.c_float, _p]
        L.or_rope_table.argtypes = [C.c_float, C.c_int, _p, _p]
        L.or_rope_axial.argtypes = [_p, _i64, _i64, _p, _p, C.c_float]
        L.or_attention.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p]
        L.or_attention_masked.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p, _p]
        L.or_attention_softmax.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p, _p, _p]
        L.or_gelu_erf.argtypes = [_p, _i64, _p]
        L.or_patch_embed.argtypes = [C.c_int, _p, _p, _p]
        L.or_trunk_run.argtypes = [_p, _p, C.c_int, _p, _p]
        L.or_set_sum_variant.argtypes = [C.c_int]
        L.or_bilinear_resize_rgb.argtypes = [_p, C.c_int, C.c_int, _p]

    def set_sum_variant(self, v: int):
        self.lib.or_set_sum_variant(v)

    def fp16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.uint16)
        self.lib.or_fp32_to_fp16_row(_ptr(x), _ptr(y), x.size)
        return y

    def dequantize(self, wtype, raw: np.ndarray, n: int):
        y = np.empty(n, np.float32)
        self.lib.or_dequantize(wtype, _ptr(np.ascontiguousarray(raw)), n, _ptr(y))
        return y

    def quantize_q8_0_act(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.size // 32 * 34, np.uint8)
        self.lib.or_quantize_q8_0_act(_ptr(x), x.size, _ptr(out))
        return out

    def round_activations(self, wtype, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.or_round_activations(wtype, _ptr(x), x.size, _ptr(y))
        return y

    def linear(self, wtype, w_raw, N, K, x, bias=None):
        x = np.ascontiguousarray(x, np.float32)
        M = x.size // K
        y = np.empty((M, N), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.lib.or_linear(wtype, _ptr(np.ascontiguousarray(w_raw)), N, K, _ptr(x), M, _ptr(b), _ptr(y))
        return y

    def layer_norm(self, x, gamma=None, beta=None, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        rows, cols = x.shape
        y = np.empty_like(x)
        g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
        b = None if beta is None else np.ascontiguousarray(beta, np.float32)
        self.lib.or_layer_norm(_ptr(x), rows, cols, _ptr(g), _ptr(b), eps, _ptr(y))
        return y

    def rope_table(self, scale, npos):
        c = np.empty((npos, 16), np.float32)
        s = np.empty((npos, 16), np.float32)
        self.lib.or_rope_table(scale, npos, _ptr(c), _ptr(s))
        return c, s

    def rope_axial(self, x, pos_x, pos_y, scale):
        x = np.array(x, np.float32, copy=True, order="C")
        tokens, heads = x.shape[0], x.shape[1]
        px = np.ascontiguousarray(pos_x, np.int32)
        py = np.ascontiguousarray(pos_y, np.int32)
        self.lib.or_rope_axial(_ptr(x), tokens, heads, _ptr(px), _ptr(py), scale)
        return x

    def attention(self, q, k, v, scale=0.125):
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        nq, heads, d = q.shape
        out = np.empty_like(q)
        self.lib.or_attention(_ptr(q), _ptr(k), _ptr(v), nq, k.shape[0], heads, d, scale, _ptr(out))
        return out

    def attention_masked(self, q, k, v, scale, key_mask=None):
        """ggml_flash_attn_ext with a per-key additive mask (-inf: key skipped;
        a row with no key left gives 0).  q [nq][heads][d], k/v [nk][heads][d]."""
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        m = None if key_mask is None else np.ascontiguousarray(key_mask, np.float32)
        nq, heads, d = q.shape
        out = np.empty_like(q)
        self.lib.or_attention_masked(_ptr(q), _ptr(k), _ptr(v), nq, k.shape[0], heads, d, scale, _ptr(m), _ptr(out))
        return out

    def attention_softmax(self, q, k, v, scale, bias=None, key_mask=None):
        """The decoder's attention (explicit ggml_soft_max_ext): bias [heads][nq][nk]
        or key_mask [nk], either optional.  q [nq][heads][d], k/v [nk][heads][d]."""
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        m = None if key_mask is None else np.ascontiguousarray(key_mask, np.float32)
        nq, heads, d = q.shape
        out = np.empty_like(q)
        self.lib.or_attention_softmax(_ptr(q), _ptr(k), _ptr(v), nq, k.shape[0], heads, d, scale, _ptr(b), _ptr(m),
                                      _ptr(out))
        return out

    def gelu_erf(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.lib.or_gelu_erf(_ptr(x), x.size, _ptr(y))
        return y

    def bilinear_resize_rgb(self, rgb):
        """uint8 [h, w, 3] -> [3, 1008, 1008] fp32 (tools/sam3_vision_trunk.cpp:33-66)."""
        src = np.ascontiguousarray(rgb, np.uint8)
        h, w = src.shape[:2]
        out = np.empty((3, 1008, 1008), np.float32)
        self.lib.or_bilinear_resize_rgb(_ptr(src), w, h, _ptr(out))
        return out

    def patch_embed(self, wtype, w_raw, image):
        img = np.ascontiguousarray(image, np.float32).reshape(3, 1008, 1008)
        out = np.empty((5184, 1024), np.float32)
        self.lib.or_patch_embed(wtype, _ptr(np.ascontiguousarray(w_raw)), _ptr(img), _ptr(out))
        return out

    def trunk(self, model: "TrunkTensors", image, n_layers: int | None = None):
        """Stem + the first n_layers blocks; returns NCHW [1, 1024, 72, 72] fp32."""
        n = model.n_layers if n_layers is None else n_layers
        img = np.ascontiguousarray(image, np.float32).reshape(3, 1008, 1008)
        out = np.empty((1, 1024, 72, 72), np.float32)
        st = model.as_struct()
        rc = self.lib.or_trunk_run(C.byref(st), _ptr(img), n, None, _ptr(out))
        if rc != 0:
            raise RuntimeError("or_trunk_run failed")
        return out


class _Layer(C.Structure):
    _fields_ = [("qkv_t", C.c_int), ("proj_t", C.c_int), ("fc1_t", C.c_int), ("fc2_t", C.c_int),
                ("qkv_w", _p), ("proj_w", _p), ("fc1_w", _p), ("fc2_w", _p),
                ("n1w", _p), ("n1b", _p), ("qkv_b", _p), ("proj_b", _p),
                ("n2w", _p), ("n2b", _p), ("fc1_b", _p), ("fc2_b", _p)]


class _Trunk(C.Structure):
    _fields_ = [("patch_t", C.c_int), ("patch_w", _p), ("pos_embed", _p), ("ln_pre_w", _p),
                ("ln_pre_b", _p), ("n_layers", C.c_int), ("layer", _Layer * 32)]


class TrunkTensors:
    """Raw trunk tensors of a GGUF file (name -> (ggml type, bytes as numpy))."""

    def __init__(self, gguf_path: str | os.PathLike):
        from gguf import GGUFReader

        path = Path(gguf_path)
        self.reader = GGUFReader(str(path))
        aliases = {}
        side = Path(str(path) + ".tensor_map.json")
        if side.exists():
            for short, orig in json.loads(side.read_text()).items():
                aliases[orig] = short
        self.t = {}
        for rt in self.reader.tensors:
            self.t[rt.name] = (int(rt.tensor_type), np.ascontiguousarray(rt.data))
        self.aliases = aliases
        self.n_layers = sum(1 for i in range(32) if self._has(f"{PREFIX}.blocks.{i}.attn.qkv.weight"))

    def _has(self, name):
        return self.aliases.get(name, name) in self.t

    def get(self, name):
        return self.t[self.aliases.get(name, name)]

    def as_struct(self) -> _Trunk:
        s = _Trunk()
        keep = []

        def raw(name):
            ty, a = self.get(name)
            keep.append(a)
            return ty, _ptr(a)

        def vec(name):
            # ensure_f32 (src/vision_trunk.cpp:35-40): 1-D tensors may be F16
            # in converted files (e.g. ln_pre.weight is not "sensitive").
            ty, a = self.get(name)
            f = np.ascontiguousarray(a.view(np.float16).astype(np.float32) if ty == F16 else a.view(np.float32))
            keep.append(f)
            return _ptr(f)

        s.patch_t, s.patch_w = raw(f"{PREFIX}.patch_embed.proj.weight")
        s.pos_embed = vec(f"{PREFIX}.pos_embed")
        s.ln_pre_w = vec(f"{PREFIX}.ln_pre.weight")
        s.ln_pre_b = vec(f"{PREFIX}.ln_pre.bias")
        s.n_layers = self.n_layers
        for i in range(self.n_layers):
            b = f"{PREFIX}.blocks.{i}"
            L = s.layer[i]
            L.qkv_t, L.qkv_w = raw(f"{b}.attn.qkv.weight")
            L.proj_t, L.proj_w = raw(f"{b}.attn.proj.weight")
            L.fc1_t, L.fc1_w = raw(f"{b}.mlp.fc1.weight")
            L.fc2_t, L.fc2_w = raw(f"{b}.mlp.fc2.weight")
            L.n1w, L.n1b = vec(f"{b}.norm1.weight"), vec(f"{b}.norm1.bias")
            L.n2w, L.n2b = vec(f"{b}.norm2.weight"), vec(f"{b}.norm2.bias")
            L.qkv_b, L.proj_b = vec(f"{b}.attn.qkv.bias"), vec(f"{b}.attn.proj.bias")
            L.fc1_b, L.fc2_b = vec(f"{b}.mlp.fc1.bias"), vec(f"{b}.mlp.fc2.bias")
        s._keep = keep  # the numpy buffers must outlive the struct
        return s


def _cpu_flags() -> set[str]:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


_ISA = re.compile(r"^(avx|amx|fma|f16c|bmi|sse|ssse|sha|vaes|vpclmul|gfni|movbe|popcnt|abm|adx|aes|pclmul|movdir|"
                  r"serialize|waitpkg|cldemote|clwb|clflushopt|rdpid|rdseed|rdrand|xsave)")


def native_build_usable(flags: set[str] | None = None) -> bool:
    """The -march=native build runs here only if this host has every ISA
    extension the build host had (recorded next to the library)."""
    rec = HERE / "_ref" / "libsam3ref_native.flags"
    if not rec.exists() or not (HERE / "_ref" / "libsam3ref_native.so").exists():
        return False
    need = {f for f in rec.read_text().split() if _ISA.match(f)}
    return need <= (flags if flags is not None else _cpu_flags())


def reference_path(prefer_native: bool = False) -> Path | None:
    """oracle/_ref build for this host: v4 (AVX-512 F/BW/DQ/VL) or v3; with
    prefer_native, the -march=native build when this host can run it (the
    reference's default GGML_NATIVE build, used for the timed CPU baseline).
    The golden fixtures were made with v4, so the checkers use v4."""
    flags = _cpu_flags()
    if prefer_native and native_build_usable(flags):
        return HERE / "_ref" / "libsam3ref_native.so"
    v4 = {"avx512f", "avx512bw", "avx512dq", "avx512vl"} <= flags
    for name in (["libsam3ref_v4.so"] if v4 else []) + ["libsam3ref_v3.so"]:
        p = HERE / "_ref" / name
        if p.exists():
            return p
    return None


def physical_cores() -> int:
    """Distinct (physical id, core id) pairs of /proc/cpuinfo: the host's
    physical cores (hyperthreads counted once)."""
    cores, phys, core = set(), "0", None
    try:
        for line in open("/proc/cpuinfo"):
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "physical id":
                phys = v
            elif k == "core id":
                core = v
            elif not k and core is not None:
                cores.add((phys, core))
                core = None
        if core is not None:
            cores.add((phys, core))
    except OSError:
        pass
    return len(cores) or (os.cpu_count() or 1)


class Reference:
    def __init__(self, path: str | os.PathLike | None = None):
        path = Path(path) if path else reference_path()
        if path is None or not Path(path).exists():
            raise FileNotFoundError("oracle/_ref not built (make -C oracle ref)")
        self.path = Path(path)
        self.lib = L = C.CDLL(str(path))
        L.ref_last_error.restype = C.c_char_p
        L.ref_trunk_run.argtypes = [C.c_char_p, _p, _p, C.c_int, C.POINTER(C.c_double)]
        L.ref_model_load.argtypes = [C.c_char_p, C.c_int]
        L.ref_model_load.restype = _p
        L.ref_model_run.argtypes = [_p, _p, _p, C.POINTER(C.c_double)]
        L.ref_model_free.argtypes = [_p]
        L.ref_mul_mat.argtypes = [C.c_int, _p, _i64, _i64, _p, _i64, _p, C.c_int]
        L.ref_norm.argtypes = [_p, _i64, _i64, C.c_float, _p]
        L.ref_rope_axial.argtypes = [_p, _i64, _i64, _p, _p, C.c_float, _p]
        L.ref_flash_attn.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p, C.c_int]
        L.ref_gelu_erf.argtypes = [_p, _i64, _p]
        L.ref_quantize_q8_0_act.argtypes = [_p, _i64, _p]
        L.ref_to_float.argtypes = [C.c_int, _p, _i64, _p]
        L.ref_fp32_to_fp16.argtypes = [_p, _i64, _p]
        L.ref_patch_embed.argtypes = [C.c_int, _p, _p, _p, C.c_int]
        if hasattr(L, "ref_bilinear_resize_rgb"):   # absent from the drop-in build
            L.ref_bilinear_resize_rgb.argtypes = [_p, C.c_int, C.c_int, _p]
        if hasattr(L, "ref_flash_attn_masked"):     # absent from the drop-in build
            L.ref_flash_attn_masked.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p, _p, C.c_int]
        if hasattr(L, "ref_decoder_mha"):
            L.ref_decoder_mha.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, C.c_float, _p, _p, _p, C.c_int]
        if hasattr(L, "ref_trunk_block"):
            L.ref_trunk_stem.argtypes = [_p, _p, _p]
            L.ref_trunk_block.argtypes = [_p, C.c_int, _p, _p]
        if hasattr(L, "ref_neck_first"):
            L.ref_neck_first.argtypes = [_p, C.c_int, _p, _p, C.POINTER(C.c_int64)]
            L.ref_neck_run.argtypes = [_p, C.c_int, _p, _p, C.POINTER(C.c_int64)]

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def trunk(self, gguf_path, image, n_threads=0):
        img = np.ascontiguousarray(image, np.float32)
        out = np.empty((1, 1024, 72, 72), np.float32)
        sec = C.c_double()
        self._check(self.lib.ref_trunk_run(str(gguf_path).encode(), _ptr(img), _ptr(out), n_threads, C.byref(sec)))
        return out, sec.value

    def load(self, gguf_path, n_threads=0) -> "RefModel":
        """The reference's GgufModel for gguf_path (CPU backend), for the
        per-block entry points."""
        h = self.lib.ref_model_load(str(gguf_path).encode(), n_threads)
        if not h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return RefModel(self, h)

    def mul_mat(self, wtype, w_raw, N, K, x, n_threads=4):
        x = np.ascontiguousarray(x, np.float32)
        M = x.size // K
        y = np.empty((M, N), np.float32)
        self._check(self.lib.ref_mul_mat(wtype, _ptr(np.ascontiguousarray(w_raw)), N, K, _ptr(x), M, _ptr(y), n_threads))
        return y

    def norm(self, x, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self.lib.ref_norm(_ptr(x), x.shape[0], x.shape[1], eps, _ptr(y)))
        return y

    def rope_axial(self, x, pos_x, pos_y, scale):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        px = np.ascontiguousarray(pos_x, np.int32)
        py = np.ascontiguousarray(pos_y, np.int32)
        self._check(self.lib.ref_rope_axial(_ptr(x), x.shape[0], x.shape[1], _ptr(px), _ptr(py), scale, _ptr(y)))
        return y

    def flash_attn(self, q, k, v, scale=0.125, n_threads=4):
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        out = np.empty_like(q)
        self._check(self.lib.ref_flash_attn(_ptr(q), _ptr(k), _ptr(v), q.shape[0], k.shape[0], q.shape[1],
                                            q.shape[2], scale, _ptr(out), n_threads))
        return out

    def flash_attn_masked(self, q, k, v, scale, key_mask=None, n_threads=4):
        """ggml_flash_attn_ext with the encoder's F16 mask: key_mask [nk] repeated
        for every query row (src/encoder_fusion.cpp:120-133)."""
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        m = None if key_mask is None else np.ascontiguousarray(key_mask, np.float32)
        out = np.empty_like(q)
        self._check(self.lib.ref_flash_attn_masked(_ptr(q), _ptr(k), _ptr(v), q.shape[0], k.shape[0], q.shape[1],
                                                   q.shape[2], scale, _ptr(m), _ptr(out), n_threads))
        return out

    def decoder_mha(self, q, k, v, scale, bias=None, key_mask=None, n_threads=4):
        """mha() of src/decoder.cpp:95-127 run by ggml: q [nq][heads][d], k/v
        [nk][heads][d], bias [heads][nq][nk] or key_mask [nk] (F16 prompt mask)."""
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        m = None if key_mask is None else np.ascontiguousarray(key_mask, np.float32)
        out = np.empty_like(q)
        self._check(self.lib.ref_decoder_mha(_ptr(q), _ptr(k), _ptr(v), q.shape[0], k.shape[0], q.shape[1],
                                             q.shape[2], scale, _ptr(b), _ptr(m), _ptr(out), n_threads))
        return out

    def gelu_erf(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self.lib.ref_gelu_erf(_ptr(x), x.size, _ptr(y)))
        return y

    def quantize_q8_0_act(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.size // 32 * 34, np.uint8)
        self._check(self.lib.ref_quantize_q8_0_act(_ptr(x), x.size, _ptr(out)))
        return out

    def to_float(self, wtype, raw, n):
        y = np.empty(n, np.float32)
        self._check(self.lib.ref_to_float(wtype, _ptr(np.ascontiguousarray(raw)), n, _ptr(y)))
        return y

    def fp16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(x.shape, np.uint16)
        self._check(self.lib.ref_fp32_to_fp16(_ptr(x), x.size, _ptr(y)))
        return y

    def bilinear_resize_rgb(self, rgb):
        src = np.ascontiguousarray(rgb, np.uint8)
        h, w = src.shape[:2]
        out = np.empty((3, 1008, 1008), np.float32)
        self._check(self.lib.ref_bilinear_resize_rgb(_ptr(src), w, h, _ptr(out)))
        return out

    def patch_embed(self, wtype, w_raw, image, n_threads=4):
        img = np.ascontiguousarray(image, np.float32)
        out = np.empty((5184, 1024), np.float32)
        self._check(self.lib.ref_patch_embed(wtype, _ptr(np.ascontiguousarray(w_raw)), _ptr(img), _ptr(out), n_threads))
        return out


class RefModel:
    """A loaded reference GgufModel: the stem and single blocks of the
    reference trunk as ggml graphs (ref_trunk_stem / ref_trunk_block)."""

    def __init__(self, ref: Reference, handle):
        self.ref, self.h = ref, handle

    def stem(self, image) -> np.ndarray:
        img = np.ascontiguousarray(image, np.float32)
        out = np.empty((5184, 1024), np.float32)
        self.ref._check(self.ref.lib.ref_trunk_stem(self.h, _ptr(img), _ptr(out)))
        return out

    def block(self, layer: int, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(5184, 1024)
        out = np.empty_like(x)
        self.ref._check(self.ref.lib.ref_trunk_block(self.h, layer, _ptr(x), _ptr(out)))
        return out

    def _neck(self, fn, level: int, trunk_nchw) -> np.ndarray:
        x = np.ascontiguousarray(trunk_nchw, np.float32).reshape(1, 1024, 72, 72)
        out = np.empty(256 * 288 * 288, np.float32)       # the largest output (level 0: 4 x 4 upsampled)
        shape = (C.c_int64 * 4)()
        self.ref._check(fn(self.h, level, _ptr(x), _ptr(out), shape))
        n = int(np.prod(list(shape)))
        return out[:n].reshape(tuple(shape))

    def neck_first(self, level: int, trunk_nchw) -> np.ndarray:
        """The first operation of neck level `level` as a ggml graph (ref_neck_first)."""
        return self._neck(self.ref.lib.ref_neck_first, level, trunk_nchw)

    def neck_run(self, level: int, trunk_nchw) -> np.ndarray:
        """sam3::VisionNeck::run for one level (ref_neck_run)."""
        return self._neck(self.ref.lib.ref_neck_run, level, trunk_nchw)

    def close(self):
        if self.h:
            self.ref.lib.ref_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
