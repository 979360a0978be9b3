"""sam3cpp_b200 — the SAM 3 ViT vision trunk on B200 (sm_100a).

Python mirror of the reference's trunk interface over the C ABI in
include/s3t.h (libs3t.so, built in-tree by ``python -m sam3cpp_b200.build``):

* ``GgufModel``   — sam3::GgufModel (include/sam3/gguf_model.h:33-66): loads a
  trunk GGUF (+ tensor_map.json sidecar) onto one GPU.
* ``VisionTrunk`` — sam3::VisionTrunk (include/sam3/vision_trunk.h:15-26):
  ``run(image_nchw, shape_nchw)`` -> ``VisionTrunkOutput(trunk_nchw,
  shape_nchw)``, with the reference's shape/size errors; ``run_batch`` is the
  batched extension (B independent images per call).

There is no CPU fallback: if libs3t.so is missing or no sm_100 GPU is
present, construction raises.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from pathlib import Path
from typing import Sequence

import numpy as np

__all__ = ["GgufModel", "VisionTrunk", "VisionTrunkOutput", "MultiTrunk", "lib", "S3TError",
           "IMAGES_ON_DEVICE", "OUTPUT_ON_DEVICE"]

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libs3t.so"
IMAGES_ON_DEVICE, OUTPUT_ON_DEVICE = 1, 2
IMAGE, DIM, GRID = 1008, 1024, 72


class S3TError(RuntimeError):
    pass


_lib = None


def lib() -> C.CDLL:
    """The loaded libs3t.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise S3TError(f"{LIB_PATH} not built: run `python -m sam3cpp_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        p, i, i64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_size_t
        L.s3t_last_error.restype = C.c_char_p
        L.s3t_create.argtypes = [i]
        L.s3t_create.restype = p
        L.s3t_destroy.argtypes = [p]
        L.s3t_set_weight.argtypes = [p, C.c_char_p, i, C.POINTER(i64), p, sz]
        L.s3t_load_gguf.argtypes = [p, C.c_char_p, C.c_char_p]
        L.s3t_gguf_inspect.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(i), C.POINTER(i)]
        L.s3t_finalize_weights.argtypes = [p]
        L.s3t_num_layers.argtypes = [p]
        L.s3t_trunk_run.argtypes = [p, p, i, p, i, p]
        L.s3t_trunk_run_layers.argtypes = [p, p, i, i, p, i, p]
        L.s3t_trunk_run_block.argtypes = [p, i, p, i, p, p]
        L.s3t_sync.argtypes = [p, p]
        L.s3t_dequantize.argtypes = [i, p, i64, p, p]
        L.s3t_weight_operand.argtypes = [i, p, i64, p, p]
        L.s3t_gemm_f16.argtypes = [i, p, p, p, i, i, i, i, i, p, p]
        L.s3t_attention.argtypes = [i, p, p, p, i, i, i, i, p, p]
        L.s3t_rope.argtypes = [i, p, i, i, i, i, p]
        L.s3t_layernorm.argtypes = [i, p, i, p, p, p, i, p]
        L.s3t_device_status.argtypes = [i]
        L.s3t_stem_noalloc.argtypes = [p, p, i, p, p]
        L.s3t_trunk_run_rgb8.argtypes = [p, p, i, i, i, p, i, p]
        L.s3t_preprocess_rgb8.argtypes = [i, p, i, i, i, p, p]
        L.s3t_trunk_profile.argtypes = [p, p, i, p, p, C.POINTER(C.c_double), C.POINTER(C.c_int)]
        L.s3t_selftest_wait_timeout.argtypes = [i, i]
        L.s3t_mha_d32.argtypes = [i, p, p, p, i, i, i, p, p, i, p]
        L.s3t_neck_first.argtypes = [p, i, p, i, p, p]
        L.s3t_neck_first_shape.argtypes = [p, i, C.POINTER(i64)]
        L.s3t_multi_create.argtypes = [C.POINTER(i), i, C.c_char_p, C.c_char_p]
        L.s3t_multi_create.restype = p
        L.s3t_multi_destroy.argtypes = [p]
        L.s3t_multi_num_devices.argtypes = [p]
        L.s3t_multi_run.argtypes = [p, p, i, p, i, p]
        L.s3t_multi_sync.argtypes = [p, p]
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise S3TError(lib().s3t_last_error().decode())


@dataclass
class VisionTrunkOutput:
    """sam3::VisionTrunkOutput: trunk_nchw fp32 [1,1024,72,72] (flattened in
    the reference; a numpy array here) and shape_nchw."""
    trunk_nchw: np.ndarray
    shape_nchw: list = field(default_factory=list)


class GgufModel:
    """Trunk weights of a GGUF file resident on one GPU (sam3::GgufModel::load,
    src/gguf_model.cpp:83-168, with the CUDA device in place of the ggml backend)."""

    def __init__(self, path: str | Path | None = None, device: int = 0, tensor_map_path: str | None = None):
        self.device = device
        self._ctx = None
        self.path = None
        if path is not None and not self.load(path, tensor_map_path=tensor_map_path):
            raise S3TError(f"failed to load model: {lib().s3t_last_error().decode()}")

    def load(self, path: str | Path, prefer_gpu: bool = True, tensor_map_path: str | None = None) -> bool:
        """Returns False on failure like the reference (message in last_error())."""
        if not prefer_gpu:
            raise S3TError("sam3cpp_b200 has no CPU path")
        self.close()
        L = lib()
        ctx = L.s3t_create(self.device)
        if not ctx:
            return False
        if L.s3t_load_gguf(ctx, str(path).encode(), tensor_map_path.encode() if tensor_map_path else None) != 0 \
                or L.s3t_finalize_weights(ctx) != 0:
            L.s3t_destroy(ctx)
            return False
        self._ctx = ctx
        self.path = Path(path)
        return True

    @classmethod
    def from_tensors(cls, tensors: dict[str, tuple[int, np.ndarray, Sequence[int]]], device: int = 0) -> "GgufModel":
        """Build from {original name: (ggml type, raw bytes as numpy, ggml ne)}."""
        m = cls(None, device)
        L = lib()
        ctx = L.s3t_create(device)
        if not ctx:
            raise S3TError(L.s3t_last_error().decode())
        try:
            for name, (ty, raw, ne) in tensors.items():
                raw = np.ascontiguousarray(raw)
                ne4 = (C.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
                check(L.s3t_set_weight(ctx, name.encode(), ty, ne4, raw.ctypes.data, raw.nbytes))
            check(L.s3t_finalize_weights(ctx))
        except Exception:
            L.s3t_destroy(ctx)
            raise
        m._ctx = ctx
        return m

    @property
    def ctx(self):
        if self._ctx is None:
            raise S3TError("model not loaded")
        return self._ctx

    @property
    def n_layers(self) -> int:
        return lib().s3t_num_layers(self.ctx)

    def close(self):
        if self._ctx is not None:
            lib().s3t_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VisionTrunk:
    """sam3::VisionTrunk over the B200 kernels (src/vision_trunk.cpp:295-488)."""

    def __init__(self, model: GgufModel):
        self.model = model

    def run(self, image_nchw, shape_nchw: Sequence[int]) -> VisionTrunkOutput:
        # Same checks and messages as src/vision_trunk.cpp:301-306.
        if list(shape_nchw) != [1, 3, IMAGE, IMAGE]:
            raise S3TError("vision trunk expects NCHW image shape [1, 3, 1008, 1008]")
        img = np.ascontiguousarray(np.asarray(image_nchw, dtype=np.float32).reshape(-1))
        if img.size != 3 * IMAGE * IMAGE:
            raise S3TError("vision trunk input payload size mismatch")
        out = self.run_batch(img.reshape(1, 3, IMAGE, IMAGE))
        return VisionTrunkOutput(out, [1, DIM, GRID, GRID])

    def run_batch(self, images: np.ndarray, n_layers: int | None = None) -> np.ndarray:
        """images [B,3,1008,1008] fp32 (host) -> [B,1024,72,72] fp32 (host)."""
        images = np.ascontiguousarray(images, dtype=np.float32)
        if images.ndim != 4 or images.shape[1:] != (3, IMAGE, IMAGE):
            raise S3TError("vision trunk expects NCHW images [B, 3, 1008, 1008]")
        b = images.shape[0]
        out = np.empty((b, DIM, GRID, GRID), np.float32)
        L = lib()
        if n_layers is None:
            check(L.s3t_trunk_run(self.model.ctx, images.ctypes.data, b, out.ctypes.data, 0, None))
        else:
            check(L.s3t_trunk_run_layers(self.model.ctx, images.ctypes.data, b, n_layers, out.ctypes.data, 0, None))
        return out

    def run_block_device(self, layer: int, x_ptr: int, batch: int, out_ptr: int, stream: int = 0) -> None:
        """Block `layer` alone on device residuals [batch*5184][1024] fp32
        (token-major): s3t_trunk_run_block.  Synchronous."""
        check(lib().s3t_trunk_run_block(self.model.ctx, layer, C.c_void_p(x_ptr), batch, C.c_void_p(out_ptr),
                                        C.c_void_p(stream) if stream else None))

    def run_rgb8(self, rgb: np.ndarray) -> np.ndarray:
        """Decoded 8-bit RGB [h, w, 3] or [B, h, w, 3] uint8 (stbi_load layout,
        host) -> [B, 1024, 72, 72] fp32: the reference's load_image_rgb resize and
        normalization (src/pipeline.cpp:45-83) on the device, then the trunk."""
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        if rgb.ndim == 3:
            rgb = rgb[None]
        if rgb.ndim != 4 or rgb.shape[3] != 3:
            raise S3TError("rgb images must be uint8 [B, height, width, 3]")
        b, h, w = rgb.shape[:3]
        out = np.empty((b, DIM, GRID, GRID), np.float32)
        check(lib().s3t_trunk_run_rgb8(self.model.ctx, rgb.ctypes.data, w, h, b, out.ctypes.data, 0, None))
        return out

    def run_rgb8_device(self, rgb_ptr: int, width: int, height: int, batch: int, out_ptr: int, stream: int = 0,
                        rgb_on_device: bool = True, output_on_device: bool = True) -> None:
        """Raw-pointer form of run_rgb8; enqueues on `stream`."""
        flags = (IMAGES_ON_DEVICE if rgb_on_device else 0) | (OUTPUT_ON_DEVICE if output_on_device else 0)
        check(lib().s3t_trunk_run_rgb8(self.model.ctx, C.c_void_p(rgb_ptr), width, height, batch,
                                       C.c_void_p(out_ptr), flags, C.c_void_p(stream) if stream else None))

    def run_device(self, images_ptr: int, batch: int, out_ptr: int, stream: int = 0, images_on_device: bool = True,
                   output_on_device: bool = True) -> None:
        """Raw-pointer form (torch data_ptr()s); enqueues on `stream`."""
        flags = (IMAGES_ON_DEVICE if images_on_device else 0) | (OUTPUT_ON_DEVICE if output_on_device else 0)
        check(lib().s3t_trunk_run(self.model.ctx, C.c_void_p(images_ptr), batch, C.c_void_p(out_ptr), flags,
                                  C.c_void_p(stream) if stream else None))

    def neck_first_shape(self, level: int) -> tuple[int, int, int, int]:
        """[1, C, H, W] of the neck level's first-operation output (one image)."""
        shape = (C.c_int64 * 4)()
        check(lib().s3t_neck_first_shape(self.model.ctx, level, shape))
        return tuple(shape)

    def neck_first_device(self, level: int, trunk_ptr: int, batch: int, out_ptr: int, stream: int = 0) -> None:
        """The first operation of neck level `level` on the trunk's device NCHW
        output (s3t_neck_first); enqueued on `stream`."""
        check(lib().s3t_neck_first(self.model.ctx, level, C.c_void_p(trunk_ptr), batch, C.c_void_p(out_ptr),
                                   C.c_void_p(stream) if stream else None))

    PROFILE_KINDS = ("stem", "qkv", "attn_windowed", "attn_global", "proj", "layernorm", "fc1", "fc2")

    def profile(self, images_ptr: int, batch: int, out_ptr: int, stream: int = 0) -> dict:
        """One eager trunk run on device buffers with a CUDA event after every
        launch: {kernel class: (summed device ms, launches)}."""
        ms = (C.c_double * 8)()
        n = (C.c_int * 8)()
        check(lib().s3t_trunk_profile(self.model.ctx, C.c_void_p(images_ptr), batch, C.c_void_p(out_ptr),
                                      C.c_void_p(stream) if stream else None, ms, n))
        return {k: (ms[i], n[i]) for i, k in enumerate(self.PROFILE_KINDS)}

    def sync(self, stream: int = 0) -> None:
        check(lib().s3t_sync(self.model.ctx, C.c_void_p(stream) if stream else None))


class MultiTrunk:
    """The trunk on several GPUs of one node (s3t_multi_*): one weight replica
    and one host thread per GPU, images sharded by image (ceil(B / n) per
    GPU), feature maps gathered to the first GPU by peer copies (device
    buffers) or copied straight to the caller's host buffer (host buffers).
    The reference has no multi-GPU path (src/gguf_model.cpp:107-120 picks one
    device)."""

    def __init__(self, path: str | Path, devices: Sequence[int], tensor_map_path: str | None = None):
        L = lib()
        devs = (C.c_int * len(devices))(*devices)
        self._h = L.s3t_multi_create(devs, len(devices), str(path).encode(),
                                     tensor_map_path.encode() if tensor_map_path else None)
        if not self._h:
            raise S3TError(L.s3t_last_error().decode())
        self.devices = list(devices)

    @property
    def n_devices(self) -> int:
        return lib().s3t_multi_num_devices(self._h)

    def run_batch(self, images: np.ndarray) -> np.ndarray:
        """images [B,3,1008,1008] fp32 (host) -> [B,1024,72,72] fp32 (host)."""
        images = np.ascontiguousarray(images, dtype=np.float32)
        if images.ndim != 4 or images.shape[1:] != (3, IMAGE, IMAGE):
            raise S3TError("vision trunk expects NCHW images [B, 3, 1008, 1008]")
        out = np.empty((images.shape[0], DIM, GRID, GRID), np.float32)
        check(lib().s3t_multi_run(self._h, images.ctypes.data, images.shape[0], out.ctypes.data, 0, None))
        return out

    def run_device(self, images_ptr: int, batch: int, out_ptr: int, stream: int = 0, images_on_device: bool = True,
                   output_on_device: bool = True) -> None:
        """Raw-pointer form; device pointers are memory of the first GPU and
        `stream` a stream of it (enqueued, see sync)."""
        flags = (IMAGES_ON_DEVICE if images_on_device else 0) | (OUTPUT_ON_DEVICE if output_on_device else 0)
        check(lib().s3t_multi_run(self._h, C.c_void_p(images_ptr), batch, C.c_void_p(out_ptr), flags,
                                  C.c_void_p(stream) if stream else None))

    def sync(self, stream: int = 0) -> None:
        check(lib().s3t_multi_sync(self._h, C.c_void_p(stream) if stream else None))

    def close(self):
        if getattr(self, "_h", None):
            lib().s3t_multi_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


MHA_BF16 = 1
MHA_OUT_F16 = 2
MHA_BIAS = 4     # key_mask is a full bias [batch][8][q_len][kv_len] (the decoder's image cross attention)


def mha_d32(device: int, q_ptr: int, k_ptr: int, v_ptr: int, batch: int, q_len: int, kv_len: int,
            key_mask_ptr: int | None, out_ptr: int, flags: int = 0, stream: int = 0) -> None:
    """Encoder-fusion multi-head attention, 8 heads of 32: mha() of
    src/encoder_fusion.cpp:63-88 (ggml_flash_attn_ext, prec F32, scale 1/sqrt(32)).

    `batch` independent sequences back to back.  Device pointers: q
    [batch][q_len][256], k/v [batch][kv_len][256] fp16 (bf16 with MHA_BF16),
    optional key_mask [batch][kv_len] fp32 added to every row's scaled scores
    (-inf: key skipped), out [batch][q_len][256] fp32 (operand type with
    MHA_OUT_F16).  A row whose keys are all masked comes out 0, as in ggml's
    CPU kernel."""
    check(lib().s3t_mha_d32(device, C.c_void_p(q_ptr), C.c_void_p(k_ptr), C.c_void_p(v_ptr), batch, q_len, kv_len,
                            C.c_void_p(key_mask_ptr) if key_mask_ptr else None, C.c_void_p(out_ptr), flags,
                            C.c_void_p(stream) if stream else None))


def preprocess_rgb8(device: int, rgb_ptr: int, width: int, height: int, batch: int, out_ptr: int,
                    stream: int = 0) -> None:
    """Device uint8 RGB [batch][height][width][3] -> device fp32 [batch][3][1008][1008],
    the reference's bilinear_resize_rgb (tools/sam3_vision_trunk.cpp:33-66), bit-exact."""
    check(lib().s3t_preprocess_rgb8(device, C.c_void_p(rgb_ptr), width, height, batch, C.c_void_p(out_ptr),
                                    C.c_void_p(stream) if stream else None))
