"""ctypes binding of libernie_b200.so (include/ernie_cuda.h), the C ABI of the B200 DiT denoiser.

This module is a thin host-side mirror of the reference's denoise / run_dit / run_block_sequence and
layer interfaces for Python callers (tests, bench.py). It raises when the CUDA library is missing:
there is no CPU path behind it.
"""
import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libernie_b200.so")
HEADER = os.path.join(ROOT, "include", "ernie_cuda.h")

OK, ERROR, OUT_OF_MEMORY = 0, -1, -100
BF16, FP32 = 0, 1
TURBO, LINEAR = 0, 1
HIDDEN, LATENT, TEXT_DIM = 4096, 128, 3072
TENSOR_WQKV, TENSOR_WO, TENSOR_WUPGATE, TENSOR_WFC2 = range(4)


class CudaError(RuntimeError):
    """A failed call: code -1 (runtime / invalid argument)."""

    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


class GpuAllocationError(CudaError):
    """Code -100: device allocation failure (the reference's GpuAllocationError)."""


_lib = None
P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
I64 = ctypes.c_int64
U64 = ctypes.c_uint64
SZ = ctypes.c_size_t


class BlockWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in ("wq", "wk", "wv", "wo", "wup", "wgate", "wfc2", "gamma_sa", "gamma_mlp",
                                 "gamma_q", "gamma_k")]


class HeadWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in ("x_embed_w", "x_embed_b", "text_proj_w", "time1_w", "time1_b", "time2_w",
                                 "time2_b", "adaln_w", "adaln_b", "final_norm_w", "final_norm_b", "final_w",
                                 "final_b")]


class TextLayerWeights(ctypes.Structure):
    _fields_ = [(n, P) for n in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "gamma_attn", "gamma_mlp")]


class Shape(ctypes.Structure):
    _fields_ = [("width", I), ("height", I), ("text_tokens", I), ("valid_text", I)]


SIGNATURES = {
    "ernie_cuda_last_error": (ctypes.c_char_p, []),
    "ernie_cuda_device_count": (I, [ctypes.POINTER(I)]),
    "ernie_cuda_context_create": (I, [I, ctypes.POINTER(P)]),
    "ernie_cuda_context_destroy": (I, [P]),
    "ernie_cuda_context_synchronize": (I, [P]),
    "ernie_cuda_context_memory": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "ernie_cuda_context_sm_count": (I, [P, ctypes.POINTER(I)]),
    "ernie_cuda_malloc": (I, [P, SZ, ctypes.POINTER(P)]),
    "ernie_cuda_free": (I, [P, P]),
    "ernie_cuda_upload": (I, [P, P, P, SZ]),
    "ernie_cuda_download": (I, [P, P, P, SZ]),
    "ernie_cuda_memset": (I, [P, P, I, SZ]),
    "ernie_cuda_event_record": (I, [P, I]),
    "ernie_cuda_event_elapsed": (I, [P, I, I, ctypes.POINTER(F)]),
    "ernie_cuda_model_create": (I, [P, I, ctypes.POINTER(P)]),
    "ernie_cuda_model_destroy": (I, [P]),
    "ernie_cuda_model_upload_block": (I, [P, I, ctypes.POINTER(BlockWeights)]),
    "ernie_cuda_model_upload_heads": (I, [P, ctypes.POINTER(HeadWeights)]),
    "ernie_cuda_model_synthesize": (I, [P, U64]),
    "ernie_cuda_model_read_tensor": (I, [P, I, I, P, SZ]),
    "ernie_cuda_model_bytes": (I, [P, ctypes.POINTER(U64)]),
    "ernie_cuda_sdpa": (I, [P, P, P, P, P, I, I, I, I, I, I, I, P]),
    "ernie_cuda_sdpa_bf16": (I, [P, P, P, P, P, I, I, I, I, P]),
    "ernie_cuda_set_attention_query_rows": (I, [P, I]),
    "ernie_cuda_attention_query_rows": (I, [P, ctypes.POINTER(I)]),
    "ernie_cuda_rmsnorm": (I, [P, P, P, I64, I, F, P]),
    "ernie_cuda_layernorm": (I, [P, P, I64, I, F, P]),
    "ernie_cuda_gelu": (I, [P, P, I64]),
    "ernie_cuda_residual_add": (I, [P, P, P, P, I64]),
    "ernie_cuda_linear_bf16": (I, [P, P, P, P, P, I, I, I]),
    "ernie_cuda_euler_step": (I, [P, P, P, F, I, I, P]),
    "ernie_cuda_finite_latent": (I, [P, P, I, I, ctypes.POINTER(I)]),
    "ernie_cuda_unpack_for_vae": (I, [P, P, P, P, I, I, P]),
    "ernie_cuda_schedule": (I, [I, I, P, P]),
    "ernie_cuda_timestep_features": (I, [F, P]),
    "ernie_cuda_dit_constants": (I, [P, I, I, I, I, I, P, P, P]),
    "ernie_cuda_session_create": (I, [P, ctypes.POINTER(Shape), I, ctypes.POINTER(P)]),
    "ernie_cuda_session_destroy": (I, [P]),
    "ernie_cuda_session_set_conditioning": (I, [P, P, P, P, P]),
    "ernie_cuda_session_tokens": (I, [P, ctypes.POINTER(I)]),
    "ernie_cuda_session_blocks": (I, [P, I, I, P, P]),
    "ernie_cuda_session_dit": (I, [P, P, F, P]),
    "ernie_cuda_session_latent": (I, [P, ctypes.POINTER(P)]),
    "ernie_cuda_session_denoise_device": (I, [P, I, I, I, I, I, ctypes.POINTER(I)]),
    "ernie_cuda_session_denoise": (I, [P, P, P, I, I, I, I, P, ctypes.POINTER(I)]),
    "ernie_cuda_session_profile": (I, [P, I, I, ctypes.POINTER(F)]),
    "ernie_cuda_session_launches_per_step": (I, [P, ctypes.POINTER(I)]),
    "ernie_cuda_finite_latent_noalloc": (I, [P, P, I, I, ctypes.POINTER(I)]),
    "ernie_cuda_initial_noise": (I, [ctypes.c_uint, I, I, P]),
    "ernie_cuda_session_create_sp": (I, [P, ctypes.POINTER(Shape), I, I, I, ctypes.POINTER(P)]),
    "ernie_cuda_sp_handle": (I, [P, P]),
    "ernie_cuda_sp_connect": (I, [P, P]),
    "ernie_cuda_sp_layout": (I, [I, I, I, I] + [ctypes.POINTER(I)] * 5),
    "ernie_cuda_text_model_create": (I, [P, I, ctypes.POINTER(P)]),
    "ernie_cuda_text_model_destroy": (I, [P]),
    "ernie_cuda_text_model_bytes": (I, [P, ctypes.POINTER(U64)]),
    "ernie_cuda_text_model_upload_layer": (I, [P, I, ctypes.POINTER(TextLayerWeights)]),
    "ernie_cuda_text_model_synthesize": (I, [P, U64]),
    "ernie_cuda_text_constants": (I, [P, I, P, P, P]),
    "ernie_cuda_text_run_blocks": (I, [P, P, I, P, P, I, I, P]),
    "ernie_cuda_text_run_blocks_device": (I, [P, P, I, P, P, I, I, P]),
    "ernie_cuda_text_embeddings": (I, [ctypes.c_char_p, P, I, I, P]),
    "ernie_cuda_model_load_safetensors": (I, [P, I, ctypes.POINTER(ctypes.c_char_p), I, I]),
    "ernie_cuda_text_model_load_safetensors": (I, [P, I, ctypes.POINTER(ctypes.c_char_p), I]),
    "ernie_cuda_vae_load_safetensors": (I, [P, ctypes.POINTER(ctypes.c_char_p), I]),
    "ernie_cuda_safetensors_count": (I, [ctypes.c_char_p, ctypes.POINTER(I)]),
    "ernie_cuda_safetensors_entry": (I, [ctypes.c_char_p, I, ctypes.c_char_p, SZ, ctypes.c_char_p,
                                         ctypes.POINTER(I64), ctypes.POINTER(I)]),
    "ernie_cuda_vae_create": (I, [P, ctypes.POINTER(P)]),
    "ernie_cuda_vae_destroy": (I, [P]),
    "ernie_cuda_vae_tensor_count": (I, [ctypes.POINTER(I)]),
    "ernie_cuda_vae_tensor_info": (I, [I, ctypes.c_char_p, SZ, ctypes.POINTER(I), ctypes.POINTER(I)]),
    "ernie_cuda_vae_upload": (I, [P, ctypes.c_char_p, P, SZ]),
    "ernie_cuda_vae_synthesize": (I, [P, U64, I]),
    "ernie_cuda_vae_bytes": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "ernie_cuda_vae_launches": (I, [P, I, I, I, ctypes.POINTER(I)]),
    "ernie_cuda_vae_profile": (I, [P, I, I, I, I, P, P]),
    "ernie_cuda_vae_decode": (I, [P, P, I, I, I, P, P, ctypes.POINTER(I)]),
    "ernie_cuda_vae_decode_device": (I, [P, P, I, I, I, P, P, ctypes.POINTER(I)]),
    "ernie_cuda_vae_encoder_create": (I, [P, ctypes.POINTER(P)]),
    "ernie_cuda_vae_encoder_destroy": (I, [P]),
    "ernie_cuda_vae_encoder_tensor_count": (I, [ctypes.POINTER(I)]),
    "ernie_cuda_vae_encoder_tensor_info": (I, [I, ctypes.c_char_p, SZ, ctypes.POINTER(I), ctypes.POINTER(I)]),
    "ernie_cuda_vae_encoder_upload": (I, [P, ctypes.c_char_p, P, SZ]),
    "ernie_cuda_vae_encoder_synthesize": (I, [P, U64, I]),
    "ernie_cuda_vae_encoder_bytes": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "ernie_cuda_vae_encoder_launches": (I, [P, I, I, I, ctypes.POINTER(I)]),
    "ernie_cuda_vae_encoder_profile": (I, [P, I, I, I, I, P, P]),
    "ernie_cuda_vae_encode": (I, [P, P, I, I, I, P, P, P, ctypes.POINTER(I)]),
    "ernie_cuda_vae_encode_device": (I, [P, P, I, I, I, P, P, P, ctypes.POINTER(I)]),
    "ernie_cuda_vae_encoder_load_safetensors": (I, [P, ctypes.POINTER(ctypes.c_char_p), I]),
    "ernie_cuda_pe_model_load_safetensors": (I, [P, I, ctypes.POINTER(ctypes.c_char_p), I]),
    "ernie_cuda_text_model_upload_head": (I, [P, P, P]),
    "ernie_cuda_text_model_synthesize_head": (I, [P, U64]),
    "ernie_cuda_pe_session_create": (I, [P, I, I, ctypes.POINTER(P)]),
    "ernie_cuda_pe_session_destroy": (I, [P]),
    "ernie_cuda_pe_session_reset": (I, [P]),
    "ernie_cuda_pe_session_position": (I, [P, ctypes.POINTER(I)]),
    "ernie_cuda_pe_session_append": (I, [P, P, P, P, I, P]),
    "ernie_cuda_pe_logits": (I, [P, P, P]),
}


def sp_layout(tokens, image, world, rank):
    """(shard rows, gathered rows, image rows, real rows, first text slot) of a sequence-parallel rank."""
    out = [I(0) for _ in range(5)]
    check(lib().ernie_cuda_sp_layout(tokens, image, world, rank, *[ctypes.byref(o) for o in out]))
    return tuple(o.value for o in out)



def declared_functions():
    """Every entry point declared in include/ernie_cuda.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ernie_cuda_\w+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with ernie-image-ncnn-vulkan_b200/build.py")
        _lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def check(rc):
    if rc == OK:
        return
    message = lib().ernie_cuda_last_error().decode(errors="replace")
    if rc == OUT_OF_MEMORY:
        raise GpuAllocationError(rc, message)
    raise CudaError(rc, message)


def ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def device_count():
    n = I(0)
    check(lib().ernie_cuda_device_count(ctypes.byref(n)))
    return n.value


# ------------------------------------------------------------------ host helpers (no GPU needed)
def schedule(steps, kind=TURBO):
    sig = np.empty(steps + 1, np.float32)
    ts = np.empty(steps, np.float32)
    check(lib().ernie_cuda_schedule(steps, kind, ptr(sig), ptr(ts)))
    return sig, ts


def timestep_features(t):
    out = np.empty(HIDDEN, np.float32)
    check(lib().ernie_cuda_timestep_features(t, ptr(out)))
    return out


def dit_constants(width, height, valid, text, token_limit=10240, freq=None):
    n = width * height + text
    cos, sin, mask = np.empty((n, 128), np.float32), np.empty((n, 128), np.float32), np.empty(n, np.float32)
    f = None if freq is None else np.ascontiguousarray(freq, np.float32)
    check(lib().ernie_cuda_dit_constants(ptr(f), width, height, valid, text, token_limit, ptr(cos), ptr(sin),
                                         ptr(mask)))
    return cos, sin, mask


# ------------------------------------------------------------------ device objects
class Buffer:
    """Device allocation owned by a Context."""

    def __init__(self, ctx, nbytes):
        self.ctx, self.nbytes = ctx, nbytes
        p = P()
        check(lib().ernie_cuda_malloc(ctx.handle, max(nbytes, 1), ctypes.byref(p)))
        self.ptr = p.value

    @property
    def c(self):
        return ctypes.c_void_p(self.ptr)

    def upload(self, array):
        array = np.ascontiguousarray(array)
        assert array.nbytes <= self.nbytes
        check(lib().ernie_cuda_upload(self.ctx.handle, self.c, ptr(array), array.nbytes))
        return self

    def download(self, shape, dtype=np.float32):
        out = np.empty(shape, dtype)
        assert out.nbytes <= self.nbytes
        check(lib().ernie_cuda_download(self.ctx.handle, ptr(out), self.c, out.nbytes))
        return out

    def zero(self):
        check(lib().ernie_cuda_memset(self.ctx.handle, self.c, 0, self.nbytes))
        return self

    def free(self):
        if self.ptr:
            lib().ernie_cuda_free(self.ctx.handle, self.c)
            self.ptr = None


class Context:
    def __init__(self, device=0):
        h = P()
        check(lib().ernie_cuda_context_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            lib().ernie_cuda_context_destroy(self.handle)
            self.handle = None

    def synchronize(self):
        check(lib().ernie_cuda_context_synchronize(self.handle))

    def buffer(self, nbytes):
        return Buffer(self, nbytes)

    def to_device(self, array):
        array = np.ascontiguousarray(array)
        return Buffer(self, array.nbytes).upload(array)

    def sm_count(self):
        n = I(0)
        check(lib().ernie_cuda_context_sm_count(self.handle, ctypes.byref(n)))
        return n.value

    def memory(self):
        f, t = U64(0), U64(0)
        check(lib().ernie_cuda_context_memory(self.handle, ctypes.byref(f), ctypes.byref(t)))
        return f.value, t.value

    def record(self, slot):
        check(lib().ernie_cuda_event_record(self.handle, slot))

    def elapsed(self, start, end):
        ms = F(0)
        check(lib().ernie_cuda_event_elapsed(self.handle, start, end, ctypes.byref(ms)))
        return ms.value

    # layer operators on numpy arrays (upload, run, download)
    def sdpa(self, q, k, v, mask=None):
        q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
        heads, nq, width = q.shape
        kv_heads, nk, _ = k.shape
        mh, mr = 1, 1
        if mask is not None:
            mask = np.ascontiguousarray(mask, np.float32)
            if mask.ndim == 3:
                mh, mr = mask.shape[0], mask.shape[1]
            elif mask.ndim == 2:
                mr = mask.shape[0]
        bq, bk, bv = self.to_device(q), self.to_device(k), self.to_device(v)
        bm = self.to_device(mask) if mask is not None else None
        out = self.buffer(q.nbytes)
        check(lib().ernie_cuda_sdpa(self.handle, bq.c, bk.c, bv.c, bm.c if bm else None, heads, kv_heads, mh, mr,
                                    nq, nk, width, out.c))
        self.synchronize()
        res = out.download(q.shape)
        for b in (bq, bk, bv, bm, out):
            if b:
                b.free()
        return res

    def _unary(self, fn, x, *args, out_shape=None):
        x = np.ascontiguousarray(x, np.float32)
        bx = self.to_device(x)
        out = self.buffer(x.nbytes)
        check(fn(self.handle, bx.c, *args, out.c))
        self.synchronize()
        res = out.download(out_shape or x.shape)
        bx.free()
        out.free()
        return res

    def rmsnorm(self, x, gamma, eps=1e-6):
        x = np.ascontiguousarray(x, np.float32)
        w = x.shape[-1]
        bg = self.to_device(np.ascontiguousarray(gamma, np.float32))
        res = self._unary(lambda h, bx, *a: lib().ernie_cuda_rmsnorm(h, bx, bg.c, *a), x, x.size // w, w, eps)
        bg.free()
        return res

    def layernorm(self, x, eps=1e-6):
        x = np.ascontiguousarray(x, np.float32)
        w = x.shape[-1]
        return self._unary(lib().ernie_cuda_layernorm, x, x.size // w, w, eps)

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        b = self.to_device(x)
        check(lib().ernie_cuda_gelu(self.handle, b.c, x.size))
        self.synchronize()
        res = b.download(x.shape)
        b.free()
        return res

    def residual_add(self, a, b):
        a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
        ba, bb, out = self.to_device(a), self.to_device(b), self.buffer(a.nbytes)
        check(lib().ernie_cuda_residual_add(self.handle, ba.c, bb.c, out.c, a.size))
        self.synchronize()
        res = out.download(a.shape)
        for x in (ba, bb, out):
            x.free()
        return res

    def linear_bf16(self, a_bits, w_bits, bias=None):
        m, k = a_bits.shape
        n = w_bits.shape[0]
        ba, bw = self.to_device(np.ascontiguousarray(a_bits, np.uint16)), self.to_device(np.ascontiguousarray(w_bits, np.uint16))
        bb = self.to_device(np.ascontiguousarray(bias, np.float32)) if bias is not None else None
        out = self.buffer(m * n * 4)
        check(lib().ernie_cuda_linear_bf16(self.handle, ba.c, bw.c, bb.c if bb else None, out.c, m, n, k))
        self.synchronize()
        res = out.download((m, n))
        for x in (ba, bw, bb, out):
            if x:
                x.free()
        return res

    def euler_step(self, sample, prediction, delta):
        sample = np.ascontiguousarray(sample, np.float32)
        _, h, w = sample.shape
        bs, bp, out = self.to_device(sample), self.to_device(np.ascontiguousarray(prediction, np.float32)), self.buffer(sample.nbytes)
        check(lib().ernie_cuda_euler_step(self.handle, bs.c, bp.c, delta, w, h, out.c))
        self.synchronize()
        res = out.download(sample.shape)
        for x in (bs, bp, out):
            x.free()
        return res

    def finite_latent(self, latent):
        latent = np.ascontiguousarray(latent, np.float32)
        _, h, w = latent.shape
        b = self.to_device(latent)
        flag = I(0)
        check(lib().ernie_cuda_finite_latent(self.handle, b.c, w, h, ctypes.byref(flag)))
        b.free()
        return bool(flag.value)

    def unpack_for_vae(self, packed, mean, variance):
        packed = np.ascontiguousarray(packed, np.float32)
        _, h, w = packed.shape
        bp, bm, bv = self.to_device(packed), self.to_device(np.ascontiguousarray(mean, np.float32)), \
            self.to_device(np.ascontiguousarray(variance, np.float32))
        out = self.buffer(32 * 4 * h * w * 4)
        check(lib().ernie_cuda_unpack_for_vae(self.handle, bp.c, bm.c, bv.c, w, h, out.c))
        self.synchronize()
        res = out.download((32, 2 * h, 2 * w))
        for x in (bp, bm, bv, out):
            x.free()
        return res


class Model:
    """Device-resident DiT weights (all blocks stay in HBM)."""

    def __init__(self, ctx, num_blocks):
        h = P()
        check(lib().ernie_cuda_model_create(ctx.handle, num_blocks, ctypes.byref(h)))
        self.handle, self.ctx, self.num_blocks = h, ctx, num_blocks

    def close(self):
        if self.handle:
            lib().ernie_cuda_model_destroy(self.handle)
            self.handle = None

    def synthesize(self, seed):
        check(lib().ernie_cuda_model_synthesize(self.handle, seed))

    def load_safetensors(self, files, num_blocks=None, heads=True):
        """Official checkpoint tensors (layers.{b}.*, and the heads) from one or more safetensors files."""
        arr, n = _paths(files)
        check(lib().ernie_cuda_model_load_safetensors(self.handle, self.num_blocks if num_blocks is None else num_blocks,
                                                      arr, n, 1 if heads else 0))

    def upload_block(self, block, mats, gammas):
        """mats: dict name -> uint16 arrays (wq, wk, wv, wo, wup, wgate, wfc2); gammas: gamma_sa, gamma_mlp,
        gamma_q, gamma_k float32 arrays."""
        keep = {k: np.ascontiguousarray(v) for k, v in {**mats, **gammas}.items()}
        w = BlockWeights(*(ptr(keep[n]) for n in ("wq", "wk", "wv", "wo", "wup", "wgate", "wfc2", "gamma_sa",
                                                  "gamma_mlp", "gamma_q", "gamma_k")))
        check(lib().ernie_cuda_model_upload_block(self.handle, block, ctypes.byref(w)))

    def upload_heads(self, tensors):
        keep = {k: np.ascontiguousarray(v) for k, v in tensors.items()}
        w = HeadWeights(*(ptr(keep[name]) for name, _ in HeadWeights._fields_))
        check(lib().ernie_cuda_model_upload_heads(self.handle, ctypes.byref(w)))

    def read_tensor(self, block, tensor, count):
        out = np.empty(count, np.uint16)
        check(lib().ernie_cuda_model_read_tensor(self.handle, block, tensor, ptr(out), out.nbytes))
        return out

    def nbytes(self):
        b = U64(0)
        check(lib().ernie_cuda_model_bytes(self.handle, ctypes.byref(b)))
        return b.value


def _paths(files):
    files = [files] if isinstance(files, (str, bytes, os.PathLike)) else list(files)
    arr = (ctypes.c_char_p * len(files))(*[os.fsencode(f) for f in files])
    return arr, len(files)


def safetensors_entries(path):
    """[(name, dtype, shape)] of one safetensors file, in name order."""
    n = I(0)
    check(lib().ernie_cuda_safetensors_count(os.fsencode(path), ctypes.byref(n)))
    out = []
    for i in range(n.value):
        name, dtype = ctypes.create_string_buffer(512), ctypes.create_string_buffer(8)
        dims, nd = (I64 * 8)(), I(0)
        check(lib().ernie_cuda_safetensors_entry(os.fsencode(path), i, name, 512, dtype, dims, ctypes.byref(nd)))
        out.append((name.value.decode(), dtype.value.decode(), tuple(dims[j] for j in range(nd.value))))
    return out


def text_embeddings(path, ids, bucket):
    """text_embeddings: rows of the [131072][3072] BF16 table (raw file or checkpoint) -> [bucket][3072] FP32."""
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.empty((bucket, 3072), np.float32)
    check(lib().ernie_cuda_text_embeddings(os.fsencode(path), ptr(ids), ids.size, bucket, ptr(out)))
    return out


def text_constants(inv_freq, bucket, mask=False):
    """text_constants: (cos [bucket][128], sin [bucket][128], causal mask [bucket][bucket] or None)."""
    f = np.ascontiguousarray(inv_freq, np.float32)
    cos, sin = np.empty((bucket, 128), np.float32), np.empty((bucket, 128), np.float32)
    m = np.empty((bucket, bucket), np.float32) if mask else None
    check(lib().ernie_cuda_text_constants(ptr(f), bucket, ptr(cos), ptr(sin), ptr(m)))
    return cos, sin, m


class TextModel:
    """Device-resident prompt-encoder layers (run_text_blocks on the B200)."""

    NAMES = ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "gamma_attn", "gamma_mlp")

    def __init__(self, ctx, num_layers=25):
        h = P()
        check(lib().ernie_cuda_text_model_create(ctx.handle, num_layers, ctypes.byref(h)))
        self.handle, self.ctx, self.num_layers = h, ctx, num_layers

    def close(self):
        if self.handle:
            lib().ernie_cuda_text_model_destroy(self.handle)
            self.handle = None

    def synthesize(self, seed):
        check(lib().ernie_cuda_text_model_synthesize(self.handle, seed))

    def load_safetensors(self, files, num_layers=None):
        """Official checkpoint tensors (language_model.model.layers.{l}.*) from one or more safetensors files."""
        arr, n = _paths(files)
        check(lib().ernie_cuda_text_model_load_safetensors(self.handle, num_layers or self.num_layers, arr, n))

    def load_pe_safetensors(self, files, num_layers=None):
        """The prompt enhancer's checkpoint (model.layers.{l}.*, model.norm, lm_head or tied embeddings)."""
        arr, n = _paths(files)
        check(lib().ernie_cuda_pe_model_load_safetensors(self.handle, num_layers or self.num_layers, arr, n))

    def synthesize_head(self, seed):
        check(lib().ernie_cuda_text_model_synthesize_head(self.handle, seed))

    def upload_head(self, norm, lm_head_bits):
        """norm [3072] float32, lm_head [131072, 3072] uint16 BF16 bits."""
        n = np.ascontiguousarray(norm, dtype=np.float32)
        w = np.ascontiguousarray(lm_head_bits, dtype=np.uint16)
        check(lib().ernie_cuda_text_model_upload_head(self.handle, ptr(n), ptr(w)))

    def upload_layer(self, layer, tensors):
        """tensors: wq, wk, wv, wo, wgate, wup, wdown as uint16 BF16 bits; gamma_attn, gamma_mlp float32."""
        keep = {k: np.ascontiguousarray(v) for k, v in tensors.items()}
        w = TextLayerWeights(*(ptr(keep[n]) for n in self.NAMES))
        check(lib().ernie_cuda_text_model_upload_layer(self.handle, layer, ctypes.byref(w)))

    def run_blocks(self, x, cos, sin, precision=BF16, layers=None):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        check(lib().ernie_cuda_text_run_blocks(self.handle, ptr(x), x.shape[0], ptr(np.ascontiguousarray(cos, np.float32)),
                                               ptr(np.ascontiguousarray(sin, np.float32)), precision,
                                               layers or self.num_layers, ptr(out)))
        return out

    def run_blocks_device(self, x_dev, bucket, cos_dev, sin_dev, out_dev, precision=BF16, layers=None):
        check(lib().ernie_cuda_text_run_blocks_device(self.handle, x_dev.c, bucket, cos_dev.c, sin_dev.c, precision,
                                                      layers or self.num_layers, out_dev.c))

    def nbytes(self):
        b = U64(0)
        check(lib().ernie_cuda_text_model_bytes(self.handle, ctypes.byref(b)))
        return b.value


def _tensor_table(prefix):
    n = I(0)
    check(getattr(lib(), prefix + "_tensor_count")(ctypes.byref(n)))
    out = []
    for i in range(n.value):
        name = ctypes.create_string_buffer(128)
        dims = (I * 4)()
        nd = I(0)
        check(getattr(lib(), prefix + "_tensor_info")(i, name, 128, dims, ctypes.byref(nd)))
        out.append((name.value.decode(), tuple(dims[j] for j in range(nd.value))))
    return out


def vae_tensors():
    """[(diffusers name, shape)] of every VAE decoder tensor the library holds, in execution order."""
    return _tensor_table("ernie_cuda_vae")


def vae_encoder_tensors():
    """[(diffusers name, shape)] of every VAE encoder tensor the library holds, in execution order."""
    return _tensor_table("ernie_cuda_vae_encoder")


class Vae:
    """Device-resident VAE decoder (decode_vae of src/vae.h on the B200)."""

    def __init__(self, ctx):
        h = P()
        check(lib().ernie_cuda_vae_create(ctx.handle, ctypes.byref(h)))
        self.handle, self.ctx = h, ctx

    def close(self):
        if self.handle:
            lib().ernie_cuda_vae_destroy(self.handle)
            self.handle = None

    def synthesize(self, seed, bf16_weights=False):
        check(lib().ernie_cuda_vae_synthesize(self.handle, seed, 1 if bf16_weights else 0))

    def load_safetensors(self, files):
        """The official VAE checkpoint's post_quant_conv.* and decoder.* tensors."""
        arr, n = _paths(files)
        check(lib().ernie_cuda_vae_load_safetensors(self.handle, arr, n))

    def upload(self, name, array):
        a = np.ascontiguousarray(array, dtype=np.float32)
        check(lib().ernie_cuda_vae_upload(self.handle, name.encode(), ptr(a), a.size))

    def nbytes(self):
        w, ws = U64(0), U64(0)
        check(lib().ernie_cuda_vae_bytes(self.handle, ctypes.byref(w), ctypes.byref(ws)))
        return w.value, ws.value

    def launches(self, width, height, precision=BF16):
        n = I(0)
        check(lib().ernie_cuda_vae_launches(self.handle, width, height, precision, ctypes.byref(n)))
        return n.value

    PROFILE_CLASSES = ("conv", "attention_gemm", "softmax", "group_norm", "upsample", "other")

    def profile(self, width, height, precision=BF16, iters=3):
        """{class: (mean ms, algorithmic work: FLOPs for conv/attention_gemm, bytes otherwise)}."""
        ms, work = np.zeros(6, np.float64), np.zeros(6, np.float64)
        check(lib().ernie_cuda_vae_profile(self.handle, width, height, precision, iters, ptr(ms), ptr(work)))
        return {c: (float(ms[i]), float(work[i])) for i, c in enumerate(self.PROFILE_CLASSES)}

    def decode(self, unpacked, precision=BF16, rgb=False):
        """unpacked [32, h, w] -> (decoded [3, 8h, 8w] FP32, rgb bytes [8h, 8w, 3] or None, nonfinite flag)."""
        u = np.ascontiguousarray(unpacked, dtype=np.float32)
        _, h, w = u.shape
        out = np.empty((3, 8 * h, 8 * w), np.float32)
        pixels = np.empty((8 * h, 8 * w, 3), np.uint8) if rgb else None
        flag = I(0)
        check(lib().ernie_cuda_vae_decode(self.handle, ptr(u), w, h, precision, ptr(out), ptr(pixels),
                                          ctypes.byref(flag)))
        return out, pixels, flag.value

    def decode_device(self, unpacked_dev, width, height, decoded_dev, precision=BF16, rgb_dev=None):
        """Asynchronous decode between device buffers (Buffer objects) on the context's stream."""
        check(lib().ernie_cuda_vae_decode_device(self.handle, unpacked_dev.c, width, height, precision,
                                                 decoded_dev.c, rgb_dev.c if rgb_dev is not None else None, None))


PE_VOCAB = 131072


class PeSession:
    """The prompt enhancer's KV-cached decoder (PeSession of src/pe_session.h) over a TextModel's layers."""

    def __init__(self, model, capacity, precision=BF16):
        h = P()
        check(lib().ernie_cuda_pe_session_create(model.handle, capacity, precision, ctypes.byref(h)))
        self.handle, self.model = h, model

    def close(self):
        if self.handle:
            lib().ernie_cuda_pe_session_destroy(self.handle)
            self.handle = None

    def reset(self):
        check(lib().ernie_cuda_pe_session_reset(self.handle))

    def position(self):
        n = I(0)
        check(lib().ernie_cuda_pe_session_position(self.handle, ctypes.byref(n)))
        return n.value

    def append(self, embedded, cos, sin):
        """embedded [rows, 3072], cos / sin [rows, 128] -> hidden [rows, 3072]."""
        x = np.ascontiguousarray(embedded, dtype=np.float32)
        c = np.ascontiguousarray(cos, dtype=np.float32)
        s = np.ascontiguousarray(sin, dtype=np.float32)
        out = np.empty_like(x)
        check(lib().ernie_cuda_pe_session_append(self.handle, ptr(x), ptr(c), ptr(s), x.shape[0], ptr(out)))
        return out

    def logits(self, hidden):
        h = np.ascontiguousarray(hidden, dtype=np.float32).reshape(-1)
        out = np.empty(PE_VOCAB, np.float32)
        check(lib().ernie_cuda_pe_logits(self.handle, ptr(h), ptr(out)))
        return out


class VaeEncoder:
    """Device-resident VAE encoder (encode_vae of src/image_encoder.h on the B200): img2img's image latent."""

    def __init__(self, ctx):
        h = P()
        check(lib().ernie_cuda_vae_encoder_create(ctx.handle, ctypes.byref(h)))
        self.handle, self.ctx = h, ctx

    def close(self):
        if self.handle:
            lib().ernie_cuda_vae_encoder_destroy(self.handle)
            self.handle = None

    def synthesize(self, seed, bf16_weights=False):
        check(lib().ernie_cuda_vae_encoder_synthesize(self.handle, seed, 1 if bf16_weights else 0))

    def load_safetensors(self, files):
        """The official VAE checkpoint's encoder.*, quant_conv.* and bn.running_* tensors."""
        arr, n = _paths(files)
        check(lib().ernie_cuda_vae_encoder_load_safetensors(self.handle, arr, n))

    def upload(self, name, array):
        a = np.ascontiguousarray(array, dtype=np.float32)
        check(lib().ernie_cuda_vae_encoder_upload(self.handle, name.encode(), ptr(a), a.size))

    def nbytes(self):
        w, ws = U64(0), U64(0)
        check(lib().ernie_cuda_vae_encoder_bytes(self.handle, ctypes.byref(w), ctypes.byref(ws)))
        return w.value, ws.value

    def launches(self, width, height, precision=BF16):
        n = I(0)
        check(lib().ernie_cuda_vae_encoder_launches(self.handle, width, height, precision, ctypes.byref(n)))
        return n.value

    PROFILE_CLASSES = ("conv", "attention_gemm", "softmax", "group_norm", "downsample", "other")

    def profile(self, width, height, precision=BF16, iters=3):
        """{class: (mean ms, algorithmic work: FLOPs for conv/attention_gemm, bytes otherwise)}."""
        ms, work = np.zeros(6, np.float64), np.zeros(6, np.float64)
        check(lib().ernie_cuda_vae_encoder_profile(self.handle, width, height, precision, iters, ptr(ms),
                                                   ptr(work)))
        return {c: (float(ms[i]), float(work[i])) for i, c in enumerate(self.PROFILE_CLASSES)}

    def encode(self, rgb, precision=BF16):
        """RGB bytes [h, w, 3] -> (mean [32, h/8, w/8], packed [128, h/16, w/16], normalized, nonfinite)."""
        x = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w, _ = x.shape
        mean = np.empty((32, h // 8, w // 8), np.float32)
        packed = np.empty((128, h // 16, w // 16), np.float32)
        normalized = np.empty_like(packed)
        flag = I(0)
        check(lib().ernie_cuda_vae_encode(self.handle, ptr(x), w, h, precision, ptr(mean), ptr(packed),
                                          ptr(normalized), ctypes.byref(flag)))
        return mean, packed, normalized, flag.value

    def encode_device(self, rgb_dev, width, height, mean_dev, packed_dev, normalized_dev, precision=BF16):
        """Asynchronous encode between device buffers (Buffer objects) on the context's stream."""
        check(lib().ernie_cuda_vae_encode_device(self.handle, rgb_dev.c, width, height, precision, mean_dev.c,
                                                 packed_dev.c, normalized_dev.c, None))


def initial_noise(seed, width, height):
    """The reference pipeline's initial latent noise [128, height, width] (mt19937 + normal_distribution)."""
    out = np.empty((128, height, width), np.float32)
    check(lib().ernie_cuda_initial_noise(seed, width, height, ptr(out)))
    return out


SP_HANDLE_BYTES = 64


class Session:
    """One request shape and precision (activations sized once, CUDA graphs cached).

    With `sp=(rank, world, exchange)` the session is one member of a Ulysses sequence-parallel group:
    `exchange(handle_bytes)` must return every member's handle in rank order (any host channel: a
    torch.distributed all_gather_object, files, MPI)."""

    def __init__(self, model, width, height, text_tokens, valid_text, precision=BF16, sp=None):
        shape = Shape(width, height, text_tokens, valid_text)
        h = P()
        if sp is None:
            check(lib().ernie_cuda_session_create(model.handle, ctypes.byref(shape), precision, ctypes.byref(h)))
        else:
            rank, world, exchange = sp
            check(lib().ernie_cuda_session_create_sp(model.handle, ctypes.byref(shape), precision, rank, world,
                                                     ctypes.byref(h)))
            mine = ctypes.create_string_buffer(SP_HANDLE_BYTES)
            try:
                check(lib().ernie_cuda_sp_handle(h, mine))
                handles = list(exchange(mine.raw))
                if len(handles) != world or any(len(x) != SP_HANDLE_BYTES for x in handles):
                    raise CudaError(f"exchange returned {len(handles)} handles for {world} members")
                check(lib().ernie_cuda_sp_connect(h, ctypes.create_string_buffer(b"".join(handles),
                                                                                 SP_HANDLE_BYTES * world)))
            except BaseException:
                lib().ernie_cuda_session_destroy(h)
                raise
        self.handle, self.model, self.ctx = h, model, model.ctx
        self.width, self.height, self.text_tokens, self.valid_text = width, height, text_tokens, valid_text
        self.tokens = width * height + text_tokens

    def close(self):
        if self.handle:
            lib().ernie_cuda_session_destroy(self.handle)
            self.handle = None

    def set_conditioning(self, text, cos, sin, mask):
        t = None if text is None else np.ascontiguousarray(text, np.float32)
        check(lib().ernie_cuda_session_set_conditioning(self.handle, ptr(t), ptr(np.ascontiguousarray(cos, np.float32)),
                                                        ptr(np.ascontiguousarray(sin, np.float32)),
                                                        ptr(np.ascontiguousarray(mask, np.float32))))

    def blocks(self, x, modulation, first=0, count=None):
        count = self.model.num_blocks - first if count is None else count
        bx = self.ctx.to_device(np.ascontiguousarray(x, np.float32))
        bm = self.ctx.to_device(np.ascontiguousarray(modulation, np.float32))
        check(lib().ernie_cuda_session_blocks(self.handle, first, count, bx.c, bm.c))
        self.ctx.synchronize()
        out = bx.download(x.shape)
        bx.free()
        bm.free()
        return out

    def dit(self, latent, timestep):
        latent = np.ascontiguousarray(latent, np.float32)
        bl = self.ctx.to_device(latent)
        out = self.ctx.buffer(latent.nbytes)
        check(lib().ernie_cuda_session_dit(self.handle, bl.c, timestep, out.c))
        res = out.download(latent.shape)
        bl.free()
        out.free()
        return res

    def latent_ptr(self):
        p = P()
        check(lib().ernie_cuda_session_latent(self.handle, ctypes.byref(p)))
        return p

    def denoise_device(self, steps, start=0, end=None, kind=TURBO, use_graph=True):
        end = steps if end is None else end
        failed = I(0)
        check(lib().ernie_cuda_session_denoise_device(self.handle, steps, start, end, kind, int(use_graph),
                                                      ctypes.byref(failed)))

    def profile(self, kernel, iters=10):
        ms = F(0)
        check(lib().ernie_cuda_session_profile(self.handle, kernel, iters, ctypes.byref(ms)))
        return ms.value

    def launches_per_step(self):
        n = I(0)
        check(lib().ernie_cuda_session_launches_per_step(self.handle, ctypes.byref(n)))
        return n.value

    def denoise(self, initial, steps, start=0, end=None, kind=TURBO, keep_predictions=False):
        initial = np.ascontiguousarray(initial, np.float32)
        end = steps if end is None else end
        out = np.empty_like(initial)
        preds = np.empty((end - start,) + initial.shape, np.float32) if keep_predictions else None
        failed = I(0)
        check(lib().ernie_cuda_session_denoise(self.handle, ptr(initial), ptr(out), steps, start, end, kind,
                                               ptr(preds), ctypes.byref(failed)))
        return (out, preds) if keep_predictions else out
