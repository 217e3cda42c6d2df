"""ctypes wrapper for libfaie2fn.so, the B200 build of the FAIE2-FlashNext decode hot path.

Mirrors flashnext/fn.py of the reference (class FN over the engine's C ABI, same method names, argument meaning
and error behaviour: a non-zero return raises RuntimeError with fn_error()). Differences: Linux CDLL instead of
the Windows DLL; the library path comes from the FN_DLL environment variable, else the in-tree build; there is no
fallback — if the library is missing the constructor raises.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DLL = os.environ.get("FN_DLL") or os.path.join(os.path.dirname(HERE), "lib", "libfaie2fn.so")
# the model shards FN.load reads when called without paths, as the reference's SH1 / SH2 (flashnext/fn.py:9-10)
SH1 = os.environ.get("FN_SHARD1")
SH2 = os.environ.get("FN_SHARD2")

P = np.ctypeslib.ndpointer
F32 = P(np.float32, flags="C_CONTIGUOUS")
I32 = P(np.int32, flags="C_CONTIGUOUS")
U8 = P(np.uint8, flags="C_CONTIGUOUS")

# symbols include/faie2fn.h declares (the CPU test-suite checks that the library exports every one)
EXPORTS = [
    "fn_error", "fn_set_device", "fn_pdl", "fn_early", "fn_bench_hot", "fn_gemv_override", "fn_gemv_waves",
    "fn_gemv_plan", "fn_test_dequant", "fn_test_gemv", "fn_bench_gemv", "fn_w_create", "fn_w_free", "fn_w_bytes",
    "fn_w_gemv", "fn_w_gemv_host", "fn_sync", "fn_test_moe", "fn_moe_create", "fn_moe_free", "fn_moe_run",
    "fn_bench_route", "fn_moe_layer_static", "fn_test_gdn", "fn_gdn_create", "fn_gdn_free", "fn_gdn_run",
    "fn_gdn_get_state", "fn_w_gemv_argmax", "fn_w_gemv_argmax_host", "fn_argmax", "fn_argmax_keys", "fn_test_argmax",
    "fn_test_gemv_argmax", "fn_ipc_alloc", "fn_ipc_open", "fn_ipc_close", "fn_ipc_free", "fn_group_create",
    "fn_group_free", "fn_w_gemv_argmax_group", "fn_moe_ep_create", "fn_moe_ep_run", "fn_w_step_host",
    "fn_embed", "fn_rmsnorm", "fn_attn_decode", "fn_step_advance", "fn_gdn_reset",
    "fn_tc_create", "fn_tc_free", "fn_tc_gemv", "fn_test_tc_gemv", "fn_bench_tc_gemv",
    "fn_embed_batch", "fn_rmsnorm_rows", "fn_attn_decode_batch", "fn_step_advance_batch", "fn_gdn_create_batch",
    "fn_gdn_run_batch", "fn_w_weights", "fn_w_prefetch_after", "fn_moe_prefetch_after", "fn_w_norm", "fn_moe_norm",
    "fn_gemv_tune", "fn_moe_var", "fn_qmma", "fn_moe_override",
    "fn_decoder_create", "fn_decoder_free", "fn_decoder_step", "fn_decoder_launches",
    "fn_load", "fn_forward", "fn_reset", "fn_free", "fn_debug_layers", "fn_use_graphs", "fn_n_past", "fn_last_ms",
    "fn_dev_gb", "fn_split", "fn_model_dims",
]


class FnLayer(C.Structure):
    """fn_layer_t (include/faie2fn.h): one layer of the decode step."""
    _fields_ = [("kind", C.c_int), ("w_in", C.c_int * 3), ("w_in_rows", C.c_int * 3), ("w_out", C.c_int),
                ("gdn", C.c_int), ("router", C.c_int), ("moe", C.c_int), ("norm1", C.c_void_p), ("norm2", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("Kc", C.c_void_p), ("Vc", C.c_void_p)]


class FnModel(C.Structure):
    """fn_model_t (include/faie2fn.h): the decode step's sizes, shared weights and device buffers."""
    _fields_ = [(n, C.c_int) for n in ("D", "nkh", "nvh", "nh", "nkv", "ne", "vocab", "max_ctx")] + [
        ("eps", C.c_float), ("embed_type", C.c_uint32), ("embed", C.c_void_p), ("head", C.c_int),
        ("final_norm", C.c_void_p), ("inv_freq", C.c_void_p), ("fuse_norm", C.c_int), ("prefetch", C.c_int)] + [
        (n, C.c_void_p) for n in ("hidden", "xnorm", "proj", "core", "Q", "att", "router_out", "logits", "tokens", "pos",
                                  "next", "prompt_len")]


class FN:
    def __init__(self, dll: str = DLL):
        if not os.path.exists(dll):
            raise FileNotFoundError(f"{dll} not built (python faie2-flashnext_b200/build.py)")
        d = self.d = C.CDLL(dll)
        self.path = dll
        d.fn_error.restype = C.c_char_p
        d.fn_set_device.argtypes = [C.c_int]
        d.fn_pdl.argtypes = [C.c_int]
        d.fn_early.argtypes = [C.c_int]
        d.fn_bench_hot.argtypes = [C.c_int]
        d.fn_gemv_override.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
        d.fn_gemv_tune.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
        d.fn_moe_var.argtypes = [C.c_int]
        d.fn_qmma.argtypes = [C.c_int]
        d.fn_moe_override.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
        d.fn_gemv_waves.argtypes = [C.c_int]
        d.fn_gemv_plan.argtypes = [C.c_uint32, C.c_int, C.c_int, I32]
        d.fn_test_dequant.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32]
        d.fn_test_gemv.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32, C.c_int, F32]
        d.fn_bench_gemv.argtypes = [C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float)]
        d.fn_w_create.argtypes = [C.c_uint32, U8, C.c_int, C.c_int]
        d.fn_w_free.argtypes = [C.c_int]
        d.fn_w_bytes.argtypes = [C.c_int]
        d.fn_w_bytes.restype = C.c_double
        d.fn_w_gemv.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        d.fn_w_gemv_host.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        d.fn_sync.argtypes = [C.c_void_p]
        vp = C.c_void_p
        d.fn_test_moe.argtypes = [C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  U8, U8, U8, U8, U8, U8, F32, F32, F32, vp, vp]
        d.fn_moe_create.argtypes = [C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, U8, U8, U8, U8, U8, U8]
        d.fn_moe_free.argtypes = [C.c_int]
        d.fn_moe_run.argtypes = [C.c_int, vp, C.c_int, vp, vp, C.c_int, C.c_int, vp]
        d.fn_bench_route.argtypes = [C.c_int, C.c_int, C.c_int, F32, C.c_int, I32, F32, C.POINTER(C.c_float)]
        d.fn_test_gdn.argtypes = [C.c_int] * 5 + [F32] * 7 + [F32, F32, F32]
        d.fn_gdn_create.argtypes = [C.c_int, C.c_int, C.c_int] + [F32] * 6
        d.fn_gdn_free.argtypes = [C.c_int]
        d.fn_gdn_run.argtypes = [C.c_int, vp, C.c_int, vp, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, vp]
        d.fn_gdn_get_state.argtypes = [C.c_int, vp, vp]
        d.fn_w_gemv_argmax.argtypes = [C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp]
        d.fn_w_gemv_argmax_host.argtypes = [C.c_int, vp, C.c_int, vp, vp, vp]
        d.fn_argmax.argtypes = [vp, C.c_int, C.c_int, C.c_int, vp, vp]
        d.fn_argmax_keys.argtypes = [vp, C.c_int, C.c_int, vp, vp]
        d.fn_test_argmax.argtypes = [F32, C.c_int, C.c_int, I32]
        d.fn_test_gemv_argmax.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32, C.c_int, vp, I32]
        d.fn_ipc_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p), C.c_char_p]
        d.fn_ipc_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        d.fn_ipc_close.argtypes = [vp]
        d.fn_ipc_free.argtypes = [vp]
        d.fn_group_create.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_void_p), C.c_size_t]
        d.fn_group_free.argtypes = [C.c_int]
        d.fn_w_gemv_argmax_group.argtypes = [C.c_int, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp,
                                             vp]
        d.fn_moe_ep_create.argtypes = [C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, U8, U8, U8,
                                       U8, U8, U8]
        d.fn_moe_ep_run.argtypes = [C.c_int, vp, C.c_int, vp, vp, C.c_int, C.c_int, vp]
        d.fn_w_step_host.argtypes = [C.c_int, I32, vp, vp, C.c_int, vp, vp]
        d.fn_embed.argtypes = [C.c_uint32, vp, C.c_int, vp, vp, vp, vp]
        d.fn_rmsnorm.argtypes = [vp, vp, vp, C.c_int, C.c_float, vp]
        d.fn_attn_decode.argtypes = [vp] * 11 + [C.c_int, C.c_int, C.c_int, C.c_float, vp]
        d.fn_step_advance.argtypes = [vp, vp, vp, vp, C.c_int, vp]
        d.fn_gdn_reset.argtypes = [C.c_int, vp]
        d.fn_w_weights.argtypes = [C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_uint64)]
        d.fn_w_prefetch_after.argtypes = [C.c_int, vp, C.c_uint64]
        d.fn_moe_prefetch_after.argtypes = [C.c_int, vp, C.c_uint64]
        d.fn_w_norm.argtypes = [C.c_int, vp, C.c_float]
        d.fn_moe_norm.argtypes = [C.c_int, vp, C.c_float]
        d.fn_tc_create.argtypes = [C.c_uint32, U8, C.c_int, C.c_int]
        d.fn_tc_free.argtypes = [C.c_int]
        d.fn_tc_gemv.argtypes = [C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, vp]
        d.fn_embed_batch.argtypes = [C.c_uint32, vp, C.c_int, vp, C.c_int, vp, vp, C.c_int, vp]
        d.fn_rmsnorm_rows.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_float, vp]
        d.fn_attn_decode_batch.argtypes = [vp, vp, vp, C.c_int] + [vp] * 8 + [C.c_int] * 4 + [C.c_float, vp]
        d.fn_step_advance_batch.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, vp]
        d.fn_gdn_create_batch.argtypes = [C.c_int, C.c_int, C.c_int, F32, F32, F32, F32, C.c_int]
        d.fn_gdn_run_batch.argtypes = [C.c_int, vp, C.c_int, vp, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, vp]
        d.fn_test_tc_gemv.argtypes = [C.c_uint32, U8, C.c_int, C.c_int, F32, C.c_int, F32]
        d.fn_bench_tc_gemv.argtypes = [C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float)]
        # the reference's model hooks, bound as its fn.py binds them (flashnext/fn.py:27-33), and the rest
        d.fn_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int]
        d.fn_forward.argtypes = [I32, C.c_int, C.c_void_p, C.c_void_p]
        d.fn_debug_layers.argtypes = [C.c_void_p]
        d.fn_dev_gb.restype = C.c_double
        d.fn_dev_gb.argtypes = [C.c_int]
        d.fn_last_ms.restype = C.c_double
        d.fn_use_graphs.argtypes = [C.c_int]
        d.fn_model_dims.argtypes = [I32]
        d.fn_free.restype = None
        d.fn_decoder_create.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        d.fn_decoder_free.argtypes = [C.c_int]
        d.fn_decoder_step.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int64]
        d.fn_decoder_launches.argtypes = [C.c_int]
        d.fn_moe_layer_static.argtypes = [C.c_uint32, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp, vp,
                                          vp, vp, C.c_int, vp, vp, C.c_int, vp]

    def check(self, rc):
        if rc != 0:
            raise RuntimeError(self.d.fn_error().decode())

    def set_device(self, dev: int):
        self.check(self.d.fn_set_device(int(dev)))

    # ---- the reference's model API (flashnext/fn.py:40-54; engine/faie2fn.cu fn_load .. fn_debug_layers) ----
    # The C symbols fn_load .. fn_free (csrc/fn_runner.cu): a GGUF model with the qwen3next tensor names on the current
    # GPU; the batched entry (forward_batch) is this layer's (runner.py BatchEngine).
    def load(self, max_ctx=32768, split=0, *, shard1=None, shard2=None, batch=0):
        """fn_load: the reference's call form load(max_ctx, split) reads SH1 / SH2 (env FN_SHARD1 / FN_SHARD2);
        shard1 / shard2 (keywords) name the GGUF file (shard2 None: one file) or its two shards; split is accepted for
        the reference's signature (every layer stays on the current GPU); batch > 0 (<= 32) also prepares
        forward_batch for that many independent sequences."""
        if shard1 is None:
            shard1, shard2 = SH1, shard2 or SH2
        if not shard1:
            raise RuntimeError("no model file: pass shard1 or set FN_SHARD1")
        if not 0 <= int(batch) <= 32:
            raise RuntimeError("batch out of range (0..32)")
        self.free()
        self.check(self.d.fn_load(str(shard1).encode(), str(shard2).encode() if shard2 else None, int(max_ctx),
                                  int(split)))
        if batch:
            from runner import BatchEngine
            try:
                self.beng = BatchEngine(self, str(shard1), str(shard2) if shard2 else None, int(max_ctx), int(batch))
            except BaseException:
                self.free()
                raise

    def dims(self):
        """{vocab, D, layers, max_ctx} of the loaded model."""
        out = np.zeros(4, np.int32)
        self.check(self.d.fn_model_dims(out))
        return dict(zip(["vocab", "D", "layers", "max_ctx"], out.tolist()))

    def reset(self):
        self.check(self.d.fn_reset())
        if getattr(self, "beng", None) is not None:
            self.beng.reset()

    def forward(self, tokens, logits=False):
        """argmax ids int32 [nt] (and logits float32 [nt, vocab] when logits=True), nt = len(tokens) in 1..8."""
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        am = np.zeros(max(1, len(t)), np.int32)
        lg = np.zeros((len(t), self.dims()["vocab"]), np.float32) if logits and self.d.fn_n_past() >= 0 else None
        self.check(self.d.fn_forward(t, len(t), lg.ctypes.data if lg is not None else None, am.ctypes.data))
        self._last_batch = False
        return (am[:len(t)], lg) if logits else am[:len(t)]

    def forward_batch(self, tokens, logits=False):
        """The batched entry for independent sequences: tokens [batch][nt] (nt 1..8) -> argmax ids int32 [batch][nt]
        (and logits float32 [batch][nt][vocab]); the sequences advance together from n_past_batch()."""
        e = getattr(self, "beng", None)
        if e is None:
            raise RuntimeError("not loaded" if self.d.fn_n_past() < 0 else "batch not loaded (load with batch > 0)")
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        am = np.zeros(t.shape, np.int32) if t.ndim == 2 else None
        lg = np.zeros(t.shape + (e.cfg["vocab"],), np.float32) if logits and t.ndim == 2 else None
        e.forward_batch(t, lg if logits else None, am)
        self._last_batch = True
        return (am, lg) if logits else am

    def n_past_batch(self) -> int:
        e = getattr(self, "beng", None)
        return e.n_past_batch if e is not None else -1

    def debug_layers(self, buf):
        """fn_debug_layers: buf float32 [layers][nt][D] (host) receives the residual after every layer of the next
        forwards (they then step eagerly); None turns it off. The buffer is kept alive here while set."""
        if buf is not None:
            a = buf
            if (not isinstance(a, np.ndarray) or a.dtype != np.float32 or a.ndim != 3 or not a.flags.c_contiguous or
                    (self.d.fn_n_past() >= 0 and (a.shape[0] != self.dims()["layers"] or a.shape[2] != self.dims()["D"]))):
                raise RuntimeError("debug buffer: float32 [layers][nt][D] expected")
        self.check(self.d.fn_debug_layers(buf.ctypes.data if buf is not None else None))
        self._dbg = buf

    def use_graphs(self, on):
        self.check(self.d.fn_use_graphs(int(bool(on))))
        if getattr(self, "beng", None) is not None:
            self.beng.use_graphs = bool(on)

    def n_past(self) -> int:
        return self.d.fn_n_past()

    def last_ms(self) -> float:
        e = getattr(self, "beng", None)
        return e.last_ms if e is not None and getattr(self, "_last_batch", False) else self.d.fn_last_ms()

    def split(self) -> int:
        return self.d.fn_split()

    def dev_gb(self, dv=0) -> float:
        """Weight bytes of the loaded model on device dv, in GB (-1 when nothing is loaded)."""
        return self.d.fn_dev_gb(int(dv))

    def free(self):
        """fn_free: release the loaded model (nothing loaded: no-op)."""
        e, self.beng = getattr(self, "beng", None), None
        if e is not None:
            e.free()
        self.d.fn_free()
        self._dbg = None

    # ---- the reference's unit-test hooks (flashnext/fn.py:56-66) ----
    def dequant(self, qtype, raw, rows, cols):
        out = np.zeros((rows, cols), np.float32)
        self.check(self.d.fn_test_dequant(int(qtype), np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), rows, cols, out))
        return out

    def gemv(self, qtype, raw, rows, cols, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None]
        nt = x.shape[0]
        y = np.zeros((nt, rows), np.float32)
        self.check(self.d.fn_test_gemv(int(qtype), np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), rows, cols,
                                       x, nt, y))
        return y

    def gemv_argmax(self, qtype, raw, rows, cols, x, logits=True):
        """(argmax [nt], y [nt][rows] or None): the lm_head GEMV with its fused argmax on GGUF rows."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None]
        nt = x.shape[0]
        y = np.zeros((nt, rows), np.float32) if logits else None
        idx = np.zeros(nt, np.int32)
        self.check(self.d.fn_test_gemv_argmax(int(qtype), np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), rows,
                                              cols, x, nt, y.ctypes.data if logits else None, idx))
        return idx, y

    def argmax(self, logits):
        """argmax [nt] of host logits [nt][n] on the GPU (k_argmax semantics)."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        if lg.ndim == 1:
            lg = lg[None]
        out = np.zeros(lg.shape[0], np.int32)
        self.check(self.d.fn_test_argmax(lg, lg.shape[1], lg.shape[0], out))
        return out

    def gemv_plan(self, qtype, rows, cols):
        out = np.zeros(7, np.int32)
        self.check(self.d.fn_gemv_plan(int(qtype), rows, cols, out))
        return dict(zip(["lpr", "gpl", "rows_per_stage", "slots", "ctas", "threads", "ldw"], out.tolist()))

    def bench_gemv(self, qtype, rows, cols, nt=1, iters=50):
        ms = C.c_float()
        self.check(self.d.fn_bench_gemv(int(qtype), rows, cols, nt, iters, C.byref(ms)))
        return ms.value

    # ---- resident weights ----
    def w_create(self, qtype, raw, rows, cols) -> int:
        h = self.d.fn_w_create(int(qtype), np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), rows, cols)
        if h < 0:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def w_free(self, h):
        self.check(self.d.fn_w_free(h))

    def w_bytes(self, h) -> float:
        return self.d.fn_w_bytes(h)

    def w_gemv(self, h, x_ptr, xs, y_ptr, ys, nt=1, flags=0, stream=0):
        """flags: 1 = add into y, 2 = early (x complete before the previous kernel started)."""
        self.check(self.d.fn_w_gemv(h, C.c_void_p(x_ptr), xs, C.c_void_p(y_ptr), ys, nt, flags, C.c_void_p(stream)))

    def w_gemv_host(self, h, x_ptr, nt, y_ptr, stream=0):
        self.check(self.d.fn_w_gemv_host(h, C.c_void_p(x_ptr), nt, C.c_void_p(y_ptr), C.c_void_p(stream)))

    def w_gemv_argmax(self, h, x_ptr, xs, y_ptr, ys, nt=1, flags=0, row0=0, index_ptr=0, keys_ptr=0, stream=0):
        """Device pointers (0 = null for y, index, keys)."""
        self.check(self.d.fn_w_gemv_argmax(h, C.c_void_p(x_ptr), xs, C.c_void_p(y_ptr or None), ys, nt, flags, row0,
                                           C.c_void_p(index_ptr or None), C.c_void_p(keys_ptr or None),
                                           C.c_void_p(stream)))

    def w_gemv_argmax_host(self, h, x_ptr, nt, y_ptr, index_ptr, stream=0):
        self.check(self.d.fn_w_gemv_argmax_host(h, C.c_void_p(x_ptr), nt, C.c_void_p(y_ptr or None),
                                                C.c_void_p(index_ptr), C.c_void_p(stream)))

    def argmax_dev(self, logits_ptr, ls, n, nt, out_ptr, stream=0):
        self.check(self.d.fn_argmax(C.c_void_p(logits_ptr), ls, n, nt, C.c_void_p(out_ptr), C.c_void_p(stream)))

    def argmax_keys(self, keys_ptr, nranks, nt, out_ptr, stream=0):
        self.check(self.d.fn_argmax_keys(C.c_void_p(keys_ptr), nranks, nt, C.c_void_p(out_ptr), C.c_void_p(stream)))

    def w_step_host(self, handles, x_ptr, y_ptr, head=-1, index_ptr=0, stream=0):
        """A decode step's GEMVs on host buffers (x / y: the inputs / outputs back to back; head: the lm_head's
        position, its argmax to index_ptr)."""
        hs = np.ascontiguousarray(handles, np.int32)
        self.check(self.d.fn_w_step_host(len(hs), hs, C.c_void_p(x_ptr), C.c_void_p(y_ptr or None), head,
                                         C.c_void_p(index_ptr or None), C.c_void_p(stream)))

    # ---- the rest of a decode step (device pointers) ----
    def embed(self, qtype, E_ptr, D, tokens_ptr, pos_ptr, h_ptr, stream=0):
        self.check(self.d.fn_embed(int(qtype), C.c_void_p(E_ptr), D, C.c_void_p(tokens_ptr), C.c_void_p(pos_ptr),
                                   C.c_void_p(h_ptr), C.c_void_p(stream)))

    def rmsnorm(self, x_ptr, w_ptr, out_ptr, D, eps=1e-6, stream=0):
        self.check(self.d.fn_rmsnorm(C.c_void_p(x_ptr), C.c_void_p(w_ptr), C.c_void_p(out_ptr), D, eps,
                                     C.c_void_p(stream)))

    def attn_decode(self, qg, k, v, wq, wk, inv_freq, Q, Kc, Vc, out, pos, nh, nkv, max_ctx, eps=1e-6, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_attn_decode(vp(qg), vp(k), vp(v), vp(wq), vp(wk), vp(inv_freq), vp(Q), vp(Kc), vp(Vc),
                                         vp(out), vp(pos), nh, nkv, max_ctx, eps, vp(stream)))

    def step_advance(self, pos, tokens, nxt, prompt_len_ptr, max_ctx, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_step_advance(vp(pos), vp(tokens), vp(nxt), vp(prompt_len_ptr), max_ctx, vp(stream)))

    def gdn_reset(self, h, stream=0):
        self.check(self.d.fn_gdn_reset(h, C.c_void_p(stream)))

    # ---- peer-memory groups (one process per GPU) ----
    def ipc_alloc(self, nbytes):
        """(device pointer, 64-byte handle) of a new zeroed buffer on the current device."""
        p = C.c_void_p()
        h = C.create_string_buffer(64)
        self.check(self.d.fn_ipc_alloc(nbytes, C.byref(p), h))
        return p.value, h.raw

    def ipc_open(self, handle: bytes):
        p = C.c_void_p()
        self.check(self.d.fn_ipc_open(handle, C.byref(p)))
        return p.value

    def ipc_close(self, ptr):
        self.check(self.d.fn_ipc_close(C.c_void_p(ptr)))

    def ipc_free(self, ptr):
        self.check(self.d.fn_ipc_free(C.c_void_p(ptr)))

    def group_create(self, rank, n, bases, nbytes):
        arr = (C.c_void_p * n)(*bases)
        g = self.d.fn_group_create(rank, n, arr, nbytes)
        if g < 1:
            raise RuntimeError(self.d.fn_error().decode())
        return g

    def group_free(self, g):
        self.check(self.d.fn_group_free(g))

    def w_gemv_argmax_group(self, h, g, x_ptr, xs, y_ptr, ys, nt, flags, row0, index_ptr, stream=0):
        self.check(self.d.fn_w_gemv_argmax_group(h, g, C.c_void_p(x_ptr), xs, C.c_void_p(y_ptr or None), ys, nt, flags,
                                                 row0, C.c_void_p(index_ptr), C.c_void_p(stream)))

    def moe_ep_create(self, gu_type, down_type, ne, k, ffe, d, group, Wg, Wu, Wd, Wsg, Wsu, Wsd):
        """Expert-parallel MoE weights of this rank (its expert slice of Wg / Wu / Wd, the whole shared expert)."""
        u8 = lambda a: np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)
        h = self.d.fn_moe_ep_create(int(gu_type), int(down_type), ne, k, ffe, d, group, u8(Wg), u8(Wu), u8(Wd), u8(Wsg),
                                    u8(Wsu), u8(Wsd))
        if h < 1:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def moe_ep_run(self, h, logits_ptr, ls, x_ptr, y_ptr, nt=1, acc=0, stream=0):
        self.check(self.d.fn_moe_ep_run(h, C.c_void_p(logits_ptr), ls, C.c_void_p(x_ptr), C.c_void_p(y_ptr), nt, acc,
                                        C.c_void_p(stream)))

    # ---- batched decode on the tensor cores (tcgen05), 1..32 tokens ----
    def tc_create(self, qtype, raw, rows, cols) -> int:
        h = self.d.fn_tc_create(int(qtype), np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), rows, cols)
        if h < 0:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def tc_free(self, h):
        self.check(self.d.fn_tc_free(h))

    def tc_gemv(self, h, x_ptr, xs, y_ptr, ys, nt, flags=0, stream=0):
        """flags: 1 = add into y."""
        vp = C.c_void_p
        self.check(self.d.fn_tc_gemv(h, vp(x_ptr), xs, vp(y_ptr), ys, nt, flags, vp(stream)))

    # ---- batched decode: independent sequences at one position ----
    def embed_batch(self, qtype, E_ptr, D, tokens_ptr, tstride, pos_ptr, h_ptr, batch, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_embed_batch(int(qtype), vp(E_ptr), D, vp(tokens_ptr), tstride, vp(pos_ptr), vp(h_ptr),
                                         batch, vp(stream)))

    def rmsnorm_rows(self, x_ptr, w_ptr, out_ptr, D, rows, eps=1e-6, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_rmsnorm_rows(vp(x_ptr), vp(w_ptr), vp(out_ptr), D, rows, eps, vp(stream)))

    def attn_decode_batch(self, qg, k, v, ss, wq, wk, inv_freq, Q, Kc, Vc, out, pos, nh, nkv, max_ctx, batch,
                          eps=1e-6, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_attn_decode_batch(vp(qg), vp(k), vp(v), ss, vp(wq), vp(wk), vp(inv_freq), vp(Q), vp(Kc),
                                               vp(Vc), vp(out), vp(pos), nh, nkv, max_ctx, batch, eps, vp(stream)))

    def step_advance_batch(self, pos, tokens, nxt, prompt_len_ptr, max_ctx, batch, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_step_advance_batch(vp(pos), vp(tokens), vp(nxt), vp(prompt_len_ptr), max_ctx, batch,
                                                vp(stream)))

    def gdn_create_batch(self, nkh, nvh, conv_w, dt_bias, ssm_a, norm_w, batch, ds=128) -> int:
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        h = self.d.fn_gdn_create_batch(nkh, nvh, ds, f(conv_w), f(dt_bias), f(ssm_a), f(norm_w), batch)
        if h < 0:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def gdn_run_batch(self, h, qkv_ptr, qs, z_ptr, zs, ab_ptr, abs_, out_ptr, os_, prefetch_state=0, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_gdn_run_batch(h, vp(qkv_ptr), qs, vp(z_ptr), zs, vp(ab_ptr), abs_, vp(out_ptr), os_,
                                           prefetch_state, vp(stream)))

    def test_tc_gemv(self, qtype, raw, rows, cols, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        y = np.zeros((x.shape[0], rows), np.float32)
        self.check(self.d.fn_test_tc_gemv(int(qtype), np.ascontiguousarray(raw, np.uint8).reshape(-1), rows, cols,
                                          x.reshape(-1), x.shape[0], y.reshape(-1)))
        return y

    def bench_tc_gemv(self, qtype, rows, cols, nt, iters=200) -> float:
        ms = C.c_float()
        self.check(self.d.fn_bench_tc_gemv(int(qtype), rows, cols, nt, iters, C.byref(ms)))
        return ms.value

    # ---- L2 prefetch hints of a decode chain ----
    def w_weights(self, h):
        """(device address, bytes) of a resident weight."""
        p, n = C.c_void_p(), C.c_uint64()
        self.check(self.d.fn_w_weights(h, C.byref(p), C.byref(n)))
        return p.value, n.value

    def w_prefetch_after(self, h, ptr, nbytes):
        self.check(self.d.fn_w_prefetch_after(h, C.c_void_p(ptr or None), nbytes))

    def moe_prefetch_after(self, h, ptr, nbytes):
        self.check(self.d.fn_moe_prefetch_after(h, C.c_void_p(ptr or None), nbytes))

    def w_norm(self, h, w_ptr, eps=1e-6):
        """RMSNorm folded into GEMV handle h (w_ptr: device norm weight; 0 turns it off)."""
        self.check(self.d.fn_w_norm(h, C.c_void_p(w_ptr or None), eps))

    def moe_norm(self, h, w_ptr, eps=1e-6):
        """RMSNorm folded into MoE layer h (w_ptr: device norm weight; 0 turns it off)."""
        self.check(self.d.fn_moe_norm(h, C.c_void_p(w_ptr or None), eps))

    def gemv_override(self, wpt=0, ks=0, tb=0, warps_per_sm=16):
        """The reference's plan override (engine/faie2fn.cu:2786-2791): tb threads per CTA (0: automatic) and the
        target warps per SM for weights created from now on; wpt and ks have no counterpart here."""
        self.d.fn_gemv_override(wpt, ks, tb, warps_per_sm)

    def gemv_tune(self, warps=-1, ring_kb=0, stage_kb=0, ctas_per_sm=0):
        """This plan's own settings for weights created from now on (warps 0 = by weight size, < 0 keeps)."""
        self.d.fn_gemv_tune(warps, ring_kb, stage_kb, ctas_per_sm)

    def moe_var(self, v):
        """MoE variant (engine/faie2fn.cu:2799): 0 = a routing kernel, 1 = routed inside the expert kernels."""
        self.d.fn_moe_var(v)

    def qmma(self, on):
        """Q4_K / Q6_K GEMVs of 1..4 tokens on the tensor cores as exact integer products (1) or not (0, default)."""
        self.d.fn_qmma(1 if on else 0)

    def sync(self, stream=0):
        self.check(self.d.fn_sync(C.c_void_p(stream)))

    # ---- MoE layer (routing + routed experts + shared expert) ----
    def moe(self, gu_type, down_type, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd, logits, x):
        """y [nt][d], sel [nt][k], w [nt][k] of one MoE layer (weights: expert-stacked GGUF rows)."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, d)
        nt = x.shape[0]
        logits = np.ascontiguousarray(logits, np.float32).reshape(nt, ne + 1)
        y = np.zeros((nt, d), np.float32)
        sel = np.zeros((nt, k), np.int32)
        w = np.zeros((nt, k), np.float32)
        u8 = lambda a: np.ascontiguousarray(a, np.uint8).reshape(-1)  # noqa: E731
        self.check(self.d.fn_test_moe(int(gu_type), int(down_type), ne, k, ffe, d, nt, u8(Wg), u8(Wu), u8(Wd), u8(Wsg),
                                      u8(Wsu), u8(Wsd), logits, x, y, sel.ctypes.data, w.ctypes.data))
        return y, sel, w

    def moe_create(self, gu_type, down_type, ne, k, ffe, d, Wg, Wu, Wd, Wsg, Wsu, Wsd) -> int:
        u8 = lambda a: np.ascontiguousarray(a, np.uint8).reshape(-1)  # noqa: E731
        h = self.d.fn_moe_create(int(gu_type), int(down_type), ne, k, ffe, d, u8(Wg), u8(Wu), u8(Wd), u8(Wsg), u8(Wsu),
                                 u8(Wsd))
        if h < 0:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def moe_free(self, h):
        self.check(self.d.fn_moe_free(h))

    def moe_run(self, h, logits_ptr, ls, x_ptr, y_ptr, nt=1, acc=0, stream=0):
        self.check(self.d.fn_moe_run(h, C.c_void_p(logits_ptr), ls, C.c_void_p(x_ptr), C.c_void_p(y_ptr), nt, acc,
                                     C.c_void_p(stream)))

    def bench_route(self, variant, part, nt, ks, iters=1):
        """flashnext/route_fn.py:20-25: routing of split-K router partials part[ks][8][528]."""
        sel = np.zeros(nt * 10, np.int32)
        w = np.zeros(nt * 10, np.float32)
        ms = C.c_float()
        self.check(self.d.fn_bench_route(variant, nt, ks, np.ascontiguousarray(part, np.float32).reshape(-1), iters, sel,
                                         w, C.byref(ms)))
        return sel, w, ms.value

    def moe_layer_static(self, gu_type, down_type, ne, k, ffe, d, w_ptrs, logits_ptr, ls, x_ptr, y_ptr, nt=1, stream=0):
        """The allocation-free MoE layer: every argument a device pointer the caller owns (w_ptrs: gate, up, down,
        shared gate, shared up, shared down)."""
        vp = C.c_void_p
        self.check(self.d.fn_moe_layer_static(int(gu_type), int(down_type), ne, k, ffe, d, *[vp(p) for p in w_ptrs],
                                              vp(logits_ptr), ls, vp(x_ptr), vp(y_ptr), nt, vp(stream)))

    # ---- gated-DeltaNet core ----
    def gdn(self, nkh, nvh, qkv, z, ab, conv_w, dt_bias, ssm_a, norm_w, S, conv_state, tokens_per_launch=1, ds=128):
        """nt tokens of the DeltaNet core; returns out [nt][nvh*ds], S and conv_state after the last token."""
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        qkv, z, ab = f(qkv), f(z), f(ab)
        nt = qkv.shape[0]
        S, cs = f(S).copy(), f(conv_state).copy()
        out = np.zeros((nt, nvh * ds), np.float32)
        self.check(self.d.fn_test_gdn(nkh, nvh, ds, nt, tokens_per_launch, qkv, z, ab, f(conv_w), f(dt_bias), f(ssm_a),
                                      f(norm_w), S, cs, out))
        return out, S, cs

    def gdn_create(self, nkh, nvh, conv_w, dt_bias, ssm_a, norm_w, S0, conv0, ds=128) -> int:
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        h = self.d.fn_gdn_create(nkh, nvh, ds, f(conv_w), f(dt_bias), f(ssm_a), f(norm_w), f(S0), f(conv0))
        if h < 0:
            raise RuntimeError(self.d.fn_error().decode())
        return h

    def gdn_free(self, h):
        self.check(self.d.fn_gdn_free(h))

    def gdn_run(self, h, qkv_ptr, qs, z_ptr, zs, ab_ptr, abs_, out_ptr, os_, nt=1, prefetch_state=0, stream=0):
        vp = C.c_void_p
        self.check(self.d.fn_gdn_run(h, vp(qkv_ptr), qs, vp(z_ptr), zs, vp(ab_ptr), abs_, vp(out_ptr), os_, nt,
                                     prefetch_state, vp(stream)))

    def gdn_state(self, h, nkh, nvh, ds=128):
        S = np.zeros((nvh, ds, ds), np.float32)
        cs = np.zeros((3, 2 * nkh * ds + nvh * ds), np.float32)
        self.check(self.d.fn_gdn_get_state(h, S.ctypes.data, cs.ctypes.data))
        return S, cs
