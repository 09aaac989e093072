"""ctypes bindings of libhxdit.so (include/hxdit.h).

The classes mirror the reference's host side: `Handle` is the FastRPC session (mega_open /
mega_close, hexagon/mega/mega_imp.c:16-18) with its rpcmem-like device buffers, `mega_block`
is the per-block call (hexagon/mega/mega.idl:10) and `chain` is megarun's block loop
(hexagon/mega/megarun.cpp:176-184). Device arrays are passed as integer device addresses;
any object with `data_ptr()` (e.g. a torch CUDA tensor) is accepted.

There is no fallback: importing works without a GPU (host helpers such as the RoPE tables run
on the CPU), but every compute entry point goes through the CUDA library and raises if it fails.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhxdit.so")

HX_OK = 0
HX_E_ARG, HX_E_CUDA, HX_E_NOWEIGHTS, HX_E_NOBLOB, HX_E_RANGE, HX_E_FORMAT, HX_E_TIMEOUT = -1, -2, -5, -6, -7, -8, -77
HX_E_SCRATCH = -9
ERRORS = {-1: "HX_E_ARG", -2: "HX_E_CUDA", -5: "HX_E_NOWEIGHTS", -6: "HX_E_NOBLOB", -7: "HX_E_RANGE",
          -8: "HX_E_FORMAT", -9: "HX_E_SCRATCH", -77: "HX_E_TIMEOUT"}

MODEL_ANIMA, MODEL_MOSS, MODEL_MOSS_PROJ = 1, 2, 3
FMT_F16, FMT_Q8, FMT_Q4A, FMT_Q4 = 0, 1, 2, 3
LORA_Q, LORA_K, LORA_V, LORA_O, LORA_UG, LORA_DN = 0, 1, 2, 3, 4, 5  # projections with rank-128 LoRA slots
EPI_STORE, EPI_RESID, EPI_GELU, EPI_RMS, EPI_SITU, EPI_STORE32 = 0, 1, 2, 3, 5, 6
(W_QKV, W_O, W_CQ, W_CKV, W_CO, W_M1, W_M2, W_Q, W_K, W_V, W_AQKV, W_AO, W_AUG, W_ADN) = range(14)
NMATS = 14

# meta slots (hexagon/mega/blk_meta.h:3-5 and moss/hexagon/mega/blk_meta.h:3-4 order)
A_SLOTS = ["X", "CTX", "MOD", "GAIN", "COS", "SIN", "WSQ", "WSK", "WSV", "WSO", "WCQ", "WCK", "WCV", "WCO", "WM1",
           "WM2", "H", "Q", "K", "V", "O", "T", "MID", "CK", "CV", "NTOK", "NCTX", "STOP", "NW", "REL", "FIRST", "Q8"]
A = {n: i for i, n in enumerate(A_SLOTS)}
A["NMETA"] = 32
A["BATCH"] = 32
A_NMETA_EXT = 33
S_SLOTS = ["X", "COS", "SIN", "H", "Q", "K", "V", "O", "T", "MID", "LQ", "LO", "LU", "LD", "NTOK", "NVALID", "STOP",
           "NW", "REL", "FIRST", "MODE", "NCB", "FMT", "ROWS", "CS", "WOFF"]
S = {n: i for i, n in enumerate(S_SLOTS)}
S["NMETA"] = 26
S["BATCH"] = 26
S["SP"] = 27
S_NMETA_EXT = 28


class HxError(RuntimeError):
    def __init__(self, rc, what):
        super().__init__(f"{what} failed: {ERRORS.get(rc, rc)} ({rc})")
        self.rc = rc


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    raise TypeError(f"expected a device address or an object with data_ptr(), got {type(x)}")


class hx_mat(ctypes.Structure):
    _fields_ = [("fmt", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int), ("group", ctypes.c_int),
                ("w", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("minv", ctypes.c_void_p)]


class hx_weight_desc(ctypes.Structure):
    _fields_ = [("model", ctypes.c_int), ("D", ctypes.c_int), ("F", ctypes.c_int), ("Cd", ctypes.c_int),
                ("H", ctypes.c_int), ("lora", ctypes.c_int), ("mats", hx_mat * NMATS), ("gain", ctypes.c_void_p),
                ("modA", ctypes.c_void_p), ("modB", ctypes.c_void_p)]


ADAPTER_BLOCK_KEYS = ("norm_sa", "sa_q", "sa_k", "sa_v", "sa_o", "sa_qn", "sa_kn", "norm_ca", "ca_q", "ca_k", "ca_v",
                      "ca_o", "ca_qn", "ca_kn", "norm_mlp", "mlp0_w", "mlp0_b", "mlp2_w", "mlp2_b")


class hx_adapter_block_desc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ADAPTER_BLOCK_KEYS]


class hx_anima_adapter_desc(ctypes.Structure):
    _fields_ = [("embed", ctypes.c_void_p), ("vocab", ctypes.c_int), ("blocks", hx_adapter_block_desc * 6),
                ("out_w", ctypes.c_void_p), ("out_b", ctypes.c_void_p), ("norm", ctypes.c_void_p)]


class hx_anima_glue_desc(ctypes.Structure):
    _fields_ = [("D", ctypes.c_int), ("t_norm", ctypes.c_void_p), ("t_lin1", ctypes.c_void_p),
                ("t_lin2", ctypes.c_void_p), ("x_emb", ctypes.c_void_p), ("f_modA", ctypes.c_void_p),
                ("f_modB", ctypes.c_void_p), ("f_lin", ctypes.c_void_p)]


class hx_moss_glue_desc(ctypes.Structure):
    _fields_ = [("D", ctypes.c_int)] + [(n, ctypes.c_void_p) for n in (
        "t_lin0", "t_b0", "t_lin2", "t_b2", "mod_w", "mod_b", "head_w", "head_b", "emb_w", "emb_b", "fin_norm",
        "fin_w", "mix_q")]


class hx_gemm_desc(ctypes.Structure):
    _fields_ = [("a", ctypes.c_void_p), ("lda", ctypes.c_int), ("a2", ctypes.c_void_p), ("lda2", ctypes.c_int),
                ("m", ctypes.c_int), ("k1", ctypes.c_int), ("w", hx_mat), ("epi", ctypes.c_int),
                ("out", ctypes.c_void_p), ("ldo", ctypes.c_int), ("x", ctypes.c_void_p), ("ldx", ctypes.c_int),
                ("gate", ctypes.c_void_p), ("vec_bstride", ctypes.c_long), ("rows_per_img", ctypes.c_int),
                ("gain0", ctypes.c_void_p), ("gain1", ctypes.c_void_p), ("seg1", ctypes.c_int),
                ("seg2", ctypes.c_int), ("rope0", ctypes.c_int), ("rope1", ctypes.c_int),
                ("cos_t", ctypes.c_void_p), ("sin_t", ctypes.c_void_p), ("eps", ctypes.c_float),
                ("tile", ctypes.c_int)]


class hx_gemm_plan(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_int), ("expand", ctypes.c_int), ("tile_m", ctypes.c_int),
                ("tile_n", ctypes.c_int), ("tiles", ctypes.c_int), ("streamk", ctypes.c_int)]


class hx_attn_desc(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("ldq", ctypes.c_int), ("q_col0", ctypes.c_int),
                ("k", ctypes.c_void_p), ("ldk", ctypes.c_int), ("k_col0", ctypes.c_int),
                ("v", ctypes.c_void_p), ("ldv", ctypes.c_int), ("v_col0", ctypes.c_int),
                ("o", ctypes.c_void_p), ("ldo", ctypes.c_int), ("batch", ctypes.c_int), ("heads", ctypes.c_int),
                ("tq", ctypes.c_int), ("tk", ctypes.c_int), ("nvalid", ctypes.c_int), ("scale", ctypes.c_float),
                ("kernel", ctypes.c_int)]


_lib = None
_vp, _i, _sz, _f, _l, _d = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_long, ctypes.c_double
_ip = ctypes.POINTER(ctypes.c_int32)
_SIGS = {
    "hx_open": [_i, ctypes.POINTER(_vp)],
    "hx_close": [_vp],
    "hx_get_stream": [_vp, ctypes.POINTER(_vp)],
    "hx_set_stream": [_vp, _vp],
    "hx_sync": [_vp],
    "hx_status": [_vp, ctypes.POINTER(_i)],
    "hx_status_ptr": [_vp, ctypes.POINTER(_vp)],
    "hx_wait_selftest": [_vp, ctypes.c_int64, _i, _ip],
    "hx_buf_alloc": [_vp, _sz, ctypes.POINTER(_i)],
    "hx_buf_free": [_vp, _i],
    "hx_buf_ptr": [_vp, _i, ctypes.POINTER(_vp)],
    "hx_buf_write": [_vp, _i, _sz, _vp, _sz],
    "hx_buf_read": [_vp, _i, _sz, _vp, _sz],
    "hx_weights_load": [_vp, _i, _vp, _sz, ctypes.POINTER(_i)],
    "hx_weights_bind": [_vp, ctypes.POINTER(hx_weight_desc), ctypes.POINTER(_i)],
    "hx_weights_free": [_vp, _i],
    "hx_lora_fold": [_vp, _i, _i, _vp, _vp, _i, _f],
    "hx_lora_fold_slots": [_vp, _i, _i, _vp, _vp, _i, _f],
    "hx_pack_apply_overlay": [_vp, _sz, _vp, _sz],
    "hx_blob_layout": [_i, _i, _i, _i, _i, _i, _i, _ip, _i, ctypes.POINTER(_sz)],
    "hx_mega_block": [_vp, _ip, _i, _i, _i, _vp, _i, _ip, _i, _ip],
    "hx_sp_unique_id": [_vp],
    "hx_sp_init": [_vp, _i, _i, _vp],
    "hx_modulation": [_vp, _i, _vp, _vp, _vp],
    "hx_modulation_noalloc": [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp],
    "hx_chain": [_vp, _ip, _i, ctypes.POINTER(_i), _i, _i, _vp, _vp, _vp, ctypes.c_uint32, _i, _ip],
    "hx_glue_load": [_vp, ctypes.POINTER(hx_anima_glue_desc), ctypes.POINTER(_i)],
    "hx_adapter_load": [_vp, ctypes.POINTER(hx_anima_adapter_desc), ctypes.POINTER(_i)],
    "hx_anima_adapter": [_vp, _i, _vp, _i, _vp, _vp, _i, _vp],
    "hx_anima_sample": [_vp, _i, _ip, _i, ctypes.POINTER(_i), _i, _i, _vp, _i, _i, _i, _vp, _i, _ip],
    "hx_moss_glue_load": [_vp, ctypes.POINTER(hx_moss_glue_desc), ctypes.POINTER(_i)],
    "hx_mgl1_tensor": [_vp, _sz, ctypes.c_char_p, ctypes.POINTER(_i), ctypes.POINTER(_i), _ip, ctypes.POINTER(_vp),
                       ctypes.POINTER(_sz)],
    "hx_moss_glue_load_mgl1": [_vp, _vp, _sz, ctypes.POINTER(_i)],
    "hx_moss_sample": [_vp, _i, _ip, _i, ctypes.POINTER(_i), _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _ip],
    "hx_gemm": [_vp, ctypes.POINTER(hx_gemm_desc)],
    "hx_attention": [_vp, ctypes.POINTER(hx_attn_desc)],
    "hx_gemm_query": [ctypes.POINTER(hx_gemm_desc), _i, ctypes.POINTER(hx_gemm_plan)],
    "hx_attention_query": [ctypes.POINTER(hx_attn_desc), _i, _ip],
    "hx_lnmod": [_vp, _vp, _vp, _i, _i, _vp, _vp, _l, _i, _f],
    "hx_rmsmod": [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _l, _i, _f],
    "hx_rope_anima": [_i, _i, _d, _i, _vp, _vp],
    "hx_rope_moss": [_i, _i, _i, _vp, _i, _vp, _vp],
    "hx_version": [],
}


def lib():
    """Load libhxdit.so (built in-tree by hexanima_b200.build); raise if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m hexanima_b200.build` (no CPU fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name == "hx_version" else ctypes.c_int
        _lib = L
    return _lib


def _check(rc, what):
    if rc != HX_OK:
        raise HxError(rc, what)


def exported_symbols():
    """Names of the functions declared in include/hxdit.h (the C ABI surface)."""
    return list(_SIGS)


def blob_layout(model, ntok, nctx, batch, D, F, Cd=1024):
    n = A_NMETA_EXT if model == MODEL_ANIMA else S_NMETA_EXT
    meta = (ctypes.c_int32 * n)()
    total = ctypes.c_size_t()
    _check(lib().hx_blob_layout(model, ntok, nctx, batch, D, F, Cd, meta, n, ctypes.byref(total)), "hx_blob_layout")
    return list(meta), total.value


def rope_anima(gh, gw, theta=10000.0, ntok=None):
    ntok = ntok or gh * gw
    c = np.zeros((ntok, 64), np.float32)
    s = np.zeros((ntok, 64), np.float32)
    _check(lib().hx_rope_anima(gh, gw, theta, ntok, c.ctypes.data, s.ctypes.data), "hx_rope_anima")
    return c, s


def rope_moss(H, W, T, bands, ntok=None):
    ntok = ntok or H * W + T
    b = np.ascontiguousarray(bands, np.float32)
    c = np.zeros((ntok, 64), np.float32)
    s = np.zeros((ntok, 64), np.float32)
    _check(lib().hx_rope_moss(H, W, T, b.ctypes.data, ntok, c.ctypes.data, s.ctypes.data), "hx_rope_moss")
    return c, s


def modulation_noalloc(modA, modB, emb, lora, mod_out, nsite, D, stream=None):
    """hx_modulation_noalloc: the per-site AdaLN modulation without a handle and without allocating;
    for callers that cannot call cudaMalloc (see include/hxdit.h). Scratch is a fixed static device array."""
    _check(lib().hx_modulation_noalloc(_ptr(modA), _ptr(modB), _ptr(emb), _ptr(lora), _ptr(mod_out), nsite, D, stream),
           "hx_modulation_noalloc")


def pack_apply_overlay(pack, ovl):
    """Apply a blkNN.ovl LoRA overlay (bytes) to a block pack held in a writable buffer (bytearray), in place."""
    pb = (ctypes.c_char * len(pack)).from_buffer(pack)
    ob = ctypes.create_string_buffer(bytes(ovl), len(ovl))
    _check(lib().hx_pack_apply_overlay(ctypes.addressof(pb), len(pack), ob, len(ovl)), "hx_pack_apply_overlay")


def mgl1_tensor(file_bytes, name):
    """A tensor of an MGL1 glue file (bytes) as a numpy array (float32 or float16), via hx_mgl1_tensor."""
    buf = ctypes.create_string_buffer(bytes(file_bytes), len(file_bytes))
    dt, nd, dims = ctypes.c_int(), ctypes.c_int(), (ctypes.c_int32 * 3)()
    data, nb = ctypes.c_void_p(), ctypes.c_size_t()
    _check(lib().hx_mgl1_tensor(buf, len(file_bytes), name.encode(), ctypes.byref(dt), ctypes.byref(nd), dims,
                                ctypes.byref(data), ctypes.byref(nb)), "hx_mgl1_tensor")
    off = data.value - ctypes.addressof(buf)
    a = np.frombuffer(bytes(file_bytes)[off:off + nb.value], np.float16 if dt.value else np.float32)
    return a.reshape(list(dims)[:nd.value]).copy()


def sp_unique_id():
    """128-byte id for hx_sp_init (create on one rank, share with all)."""
    buf = ctypes.create_string_buffer(128)
    _check(lib().hx_sp_unique_id(buf), "hx_sp_unique_id")
    return buf.raw


def make_mat(fmt, n, k, w, scale=None, minv=None, group=None):
    if group is None:
        group = 64 if fmt == FMT_F16 else 32
    return hx_mat(fmt, n, k, group, _ptr(w), _ptr(scale), _ptr(minv))


# stand-in addresses for the host-side queries: 256-byte aligned, never dereferenced
_QADDR = 1 << 20


def gemm_query(m, n, k, fmt, epi, group=None, tile=0, sm_count=148, k1=0):
    """What hx_gemm would run for an m x n x k GEMM (weights of format `fmt`, epilogue `epi`) on a GPU with
    `sm_count` SMs: dict(kernel, expand, tile_m, tile_n, tiles, streamk); kernel 1 single-CTA, 2 CTA pair,
    3 q8 weights in TMEM. Host-side only (no handle, no device)."""
    if group is None:
        group = 64 if fmt == FMT_F16 else 32
    mat = hx_mat(fmt, n, k, group, _QADDR, _QADDR, _QADDR)
    out_cols = n // 2 if epi == EPI_SITU else n
    d = hx_gemm_desc(_QADDR, k, _QADDR if k1 else None, k - k1 if k1 else 0, m, k1, mat, epi, _QADDR, out_cols,
                     _QADDR, n, _QADDR, 0, 0, _QADDR, _QADDR, n, n, 0, 0, None, None, 1e-6, tile)
    plan = hx_gemm_plan()
    _check(lib().hx_gemm_query(ctypes.byref(d), sm_count, ctypes.byref(plan)), "hx_gemm_query")
    return {f: getattr(plan, f) for f, _ in hx_gemm_plan._fields_}


def attention_query(batch, heads, tq, tk, kernel=0, sm_count=148, o_addr=_QADDR):
    """The kernel hx_attention would run (1 general, 2 short-key) for these sizes; host-side only."""
    D = 128 * heads
    d = hx_attn_desc(_QADDR, 3 * D, 0, _QADDR, 2 * D, 0, _QADDR, 2 * D, D, o_addr, D, batch, heads, tq, tk, 0, 1.0,
                     kernel)
    out = ctypes.c_int32()
    _check(lib().hx_attention_query(ctypes.byref(d), sm_count, ctypes.byref(out)), "hx_attention_query")
    return out.value


class Handle:
    """One device session: stream, status word, device buffers and weight sets."""

    def __init__(self, device=0):
        self.h = ctypes.c_void_p()
        _check(lib().hx_open(device, ctypes.byref(self.h)), "hx_open")
        self._keep = []

    def close(self):
        if self.h:
            _check(lib().hx_close(self.h), "hx_close")
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -------------------------------------------------------------- stream / status
    def stream(self):
        s = ctypes.c_void_p()
        _check(lib().hx_get_stream(self.h, ctypes.byref(s)), "hx_get_stream")
        return s.value

    def set_stream(self, stream_ptr):
        _check(lib().hx_set_stream(self.h, stream_ptr), "hx_set_stream")

    def sync(self):
        _check(lib().hx_sync(self.h), "hx_sync")

    def status(self):
        st = ctypes.c_int()
        _check(lib().hx_status(self.h, ctypes.byref(st)), "hx_status")
        return st.value

    def wait_selftest(self, limit_ns, arrive):
        """hx_wait_selftest: one bounded device wait with a run-time limit; returns its rc (HX_OK, or
        HX_E_TIMEOUT when nothing arrived within limit_ns)."""
        rc = ctypes.c_int32()
        _check(lib().hx_wait_selftest(self.h, int(limit_ns), 1 if arrive else 0, ctypes.byref(rc)), "hx_wait_selftest")
        return rc.value

    # -------------------------------------------------------------- buffers
    def buf_alloc(self, nbytes):
        fd = ctypes.c_int()
        _check(lib().hx_buf_alloc(self.h, nbytes, ctypes.byref(fd)), "hx_buf_alloc")
        return fd.value

    def buf_free(self, fd):
        _check(lib().hx_buf_free(self.h, fd), "hx_buf_free")

    def buf_ptr(self, fd):
        p = ctypes.c_void_p()
        _check(lib().hx_buf_ptr(self.h, fd, ctypes.byref(p)), "hx_buf_ptr")
        return p.value

    def buf_write(self, fd, off, arr):
        a = np.ascontiguousarray(arr)
        _check(lib().hx_buf_write(self.h, fd, off, a.ctypes.data, a.nbytes), "hx_buf_write")

    def buf_read(self, fd, off, nbytes):
        out = np.empty(nbytes, np.uint8)
        _check(lib().hx_buf_read(self.h, fd, off, out.ctypes.data, nbytes), "hx_buf_read")
        return out

    # -------------------------------------------------------------- weights
    def weights_load(self, model, pack_bytes):
        b = np.frombuffer(pack_bytes, np.uint8) if isinstance(pack_bytes, (bytes, bytearray)) else pack_bytes
        b = np.ascontiguousarray(b)
        wfd = ctypes.c_int()
        _check(lib().hx_weights_load(self.h, model, b.ctypes.data, b.nbytes, ctypes.byref(wfd)), "hx_weights_load")
        return wfd.value

    def weights_bind(self, model, D, F, mats, gain, Cd=0, H=0, lora=0, modA=None, modB=None, keep=()):
        d = hx_weight_desc()
        d.model, d.D, d.F, d.Cd, d.H, d.lora = model, D, F, Cd, H, lora
        for slot, m in mats.items():
            d.mats[slot] = m
        d.gain, d.modA, d.modB = _ptr(gain), _ptr(modA), _ptr(modB)
        wfd = ctypes.c_int()
        _check(lib().hx_weights_bind(self.h, ctypes.byref(d), ctypes.byref(wfd)), "hx_weights_bind")
        self._keep.append(keep)  # the caller's device arrays must outlive the binding
        return wfd.value

    def sp_init(self, nranks, rank, id128):
        buf = ctypes.create_string_buffer(bytes(id128), 128)
        _check(lib().hx_sp_init(self.h, nranks, rank, buf), "hx_sp_init")

    def weights_free(self, wfd):
        _check(lib().hx_weights_free(self.h, wfd), "hx_weights_free")

    def lora_fold(self, wfd, slot, B_dev, A_dev, rank, scale=1.0):
        """Fold scale * B[N][rank] @ A[rank][K_base] (device fp32) into the q8 matrix `slot` of wfd, in place."""
        _check(lib().hx_lora_fold(self.h, wfd, slot, _ptr(B_dev), _ptr(A_dev), rank, scale), "hx_lora_fold")

    def lora_fold_slots(self, wfd, proj, B_dev, A_dev, rank, scale=1.0):
        """Fold scale * B[N][rank] @ A[rank][K_base] (device fp32, B in logical row order) into the rank-128
        LoRA slots of MOSS projection `proj` (LORA_Q .. LORA_DN): best rank-128 approximation, requantised."""
        _check(lib().hx_lora_fold_slots(self.h, wfd, proj, _ptr(B_dev), _ptr(A_dev), rank, scale),
               "hx_lora_fold_slots")

    # -------------------------------------------------------------- block / chain
    def mega_block(self, meta, wfd, bfd, mod=None, ntimes=0):
        m = (ctypes.c_int32 * len(meta))(*meta)
        times = (ctypes.c_int32 * max(ntimes, 1))()
        rc = ctypes.c_int32()
        if mod is not None:
            mv = np.ascontiguousarray(mod, np.float32)
            mp, ml = mv.ctypes.data, mv.nbytes
        else:
            mp, ml = None, 0
        r = lib().hx_mega_block(self.h, m, len(meta), wfd, bfd, mp, ml, times, ntimes, ctypes.byref(rc))
        _check(r, "hx_mega_block")
        _check(rc.value, "hx_mega_block rc")
        return list(times)[:ntimes]

    def modulation(self, wfd, emb_dev, lora_dev, mod_dev):
        _check(lib().hx_modulation(self.h, wfd, _ptr(emb_dev), _ptr(lora_dev), _ptr(mod_dev)), "hx_modulation")

    def chain(self, meta, wfds, bfd, mods_dev=None, emb_dev=None, lora_dev=None, skipmask=0, use_graph=True):
        m = (ctypes.c_int32 * len(meta))(*meta)
        w = (ctypes.c_int * len(wfds))(*wfds)
        rc = ctypes.c_int32()
        r = lib().hx_chain(self.h, m, len(meta), w, len(wfds), bfd, _ptr(mods_dev), _ptr(emb_dev), _ptr(lora_dev),
                           skipmask, 1 if use_graph else 0, ctypes.byref(rc))
        _check(r, "hx_chain")
        _check(rc.value, "hx_chain rc")

    # -------------------------------------------------------------- glue + sampler
    def glue_load(self, D, t_norm, t_lin1, t_lin2, x_emb, f_modA, f_modB, f_lin):
        d = hx_anima_glue_desc(D, _ptr(t_norm), _ptr(t_lin1), _ptr(t_lin2), _ptr(x_emb), _ptr(f_modA), _ptr(f_modB),
                               _ptr(f_lin))
        g = ctypes.c_int()
        _check(lib().hx_glue_load(self.h, ctypes.byref(d), ctypes.byref(g)), "hx_glue_load")
        return g.value

    def adapter_load(self, W):
        """W: device fp16 tensors {"embed" [vocab][1024], "blocks": 6 dicts of ADAPTER_BLOCK_KEYS, "out_w", "out_b",
        "norm"} (copied into handle-owned memory)."""
        d = hx_anima_adapter_desc()
        d.embed = _ptr(W["embed"])
        d.vocab = int(W["embed"].shape[0])
        for i, b in enumerate(W["blocks"]):
            for k in ADAPTER_BLOCK_KEYS:
                setattr(d.blocks[i], k, _ptr(b[k]))
        d.out_w, d.out_b, d.norm = _ptr(W["out_w"]), _ptr(W["out_b"]), _ptr(W["norm"])
        a = ctypes.c_int()
        _check(lib().hx_adapter_load(self.h, ctypes.byref(d), ctypes.byref(a)), "hx_adapter_load")
        return a.value

    def anima_adapter(self, afd, hidden_dev, ids, wts, out_dev):
        """Context [512][1024] fp32 into out_dev from hidden_dev fp32 [S][1024] and host ids / wts [L]."""
        ids = np.ascontiguousarray(ids, np.int32)
        wts = np.ascontiguousarray(wts, np.float32)
        S = int(hidden_dev.shape[0])
        _check(lib().hx_anima_adapter(self.h, afd, _ptr(hidden_dev), S, ids.ctypes.data, wts.ctypes.data, len(ids),
                                      _ptr(out_dev)), "hx_anima_adapter")

    def anima_sample(self, gfd, meta, wfds, bfd, latent_dev, lat_h, lat_w, nsteps=4, sigmas=None, use_graph=True):
        m = (ctypes.c_int32 * len(meta))(*meta)
        w = (ctypes.c_int * len(wfds))(*wfds)
        rc = ctypes.c_int32()
        sg = None
        if sigmas is not None:
            sarr = np.ascontiguousarray(sigmas, np.float32)
            sg = sarr.ctypes.data
        r = lib().hx_anima_sample(self.h, gfd, m, len(meta), w, len(wfds), bfd, _ptr(latent_dev), lat_h, lat_w, nsteps,
                                  sg, 1 if use_graph else 0, ctypes.byref(rc))
        _check(r, "hx_anima_sample")
        _check(rc.value, "hx_anima_sample rc")

    # -------------------------------------------------------------- operators
    def moss_glue_load(self, D, **arrays):
        """MOSS sampler glue from device arrays named as the hx_moss_glue_desc fields (copied by the library)."""
        d = hx_moss_glue_desc()
        d.D = D
        for name, _ in hx_moss_glue_desc._fields_[1:]:
            setattr(d, name, _ptr(arrays[name]))
        gfd = ctypes.c_int()
        _check(lib().hx_moss_glue_load(self.h, ctypes.byref(d), ctypes.byref(gfd)), "hx_moss_glue_load")
        return gfd.value

    def moss_glue_load_mgl1(self, file_bytes):
        buf = ctypes.create_string_buffer(bytes(file_bytes), len(file_bytes))
        gfd = ctypes.c_int()
        _check(lib().hx_moss_glue_load_mgl1(self.h, buf, len(file_bytes), ctypes.byref(gfd)), "hx_moss_glue_load_mgl1")
        return gfd.value

    def moss_sample(self, gfd, meta, wfds, bfd, z_dev, x0_dev, lat_h, lat_w, text_dev, ntext, codes, use_graph=True):
        m = (ctypes.c_int32 * len(meta))(*meta)
        w = (ctypes.c_int * len(wfds))(*wfds)
        c = np.ascontiguousarray(codes, np.float32)
        rc = ctypes.c_int32()
        r = lib().hx_moss_sample(self.h, gfd, m, len(meta), w, len(wfds), bfd, _ptr(z_dev), _ptr(x0_dev), lat_h, lat_w,
                                 _ptr(text_dev), ntext, len(c), c.ctypes.data, 1 if use_graph else 0, ctypes.byref(rc))
        _check(r, "hx_moss_sample")
        _check(rc.value, "hx_moss_sample rc")

    def gemm(self, a, m, mat, epi=EPI_STORE, lda=None, k1=0, a2=None, lda2=0, out=None, ldo=0, x=None, ldx=0,
             gate=None, vec_bstride=0, rows_per_img=0, gain0=None, gain1=None, seg1=0, seg2=0, rope0=0, rope1=0,
             cos_t=None, sin_t=None, eps=1e-6, tile=0):
        d = hx_gemm_desc(_ptr(a), lda if lda is not None else mat.k, _ptr(a2), lda2, m, k1, mat, epi, _ptr(out), ldo,
                         _ptr(x), ldx, _ptr(gate), vec_bstride, rows_per_img, _ptr(gain0), _ptr(gain1), seg1, seg2,
                         rope0, rope1, _ptr(cos_t), _ptr(sin_t), eps, tile)
        _check(lib().hx_gemm(self.h, ctypes.byref(d)), "hx_gemm")

    def attention(self, q, k, v, o, batch, heads, tq, tk, ldq, ldk, ldv, ldo, q_col0=0, k_col0=0, v_col0=0,
                  nvalid=0, scale=1.0, kernel=0):
        d = hx_attn_desc(_ptr(q), ldq, q_col0, _ptr(k), ldk, k_col0, _ptr(v), ldv, v_col0, _ptr(o), ldo, batch,
                         heads, tq, tk, nvalid, scale, kernel)
        _check(lib().hx_attention(self.h, ctypes.byref(d)), "hx_attention")

    def lnmod(self, x, h16, rows, D, shift, scale, vec_bstride=0, rows_per_img=0, eps=1e-6):
        _check(lib().hx_lnmod(self.h, _ptr(x), _ptr(h16), rows, D, _ptr(shift), _ptr(scale), vec_bstride,
                              rows_per_img, eps), "hx_lnmod")

    def rmsmod(self, x, h16, rows, D, w, shift, scale, vec_bstride=0, rows_per_img=0, eps=1e-6):
        _check(lib().hx_rmsmod(self.h, _ptr(x), _ptr(h16), rows, D, _ptr(w), _ptr(shift), _ptr(scale), vec_bstride,
                               rows_per_img, eps), "hx_rmsmod")


def version():
    return lib().hx_version().decode()
