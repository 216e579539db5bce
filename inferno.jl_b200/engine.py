"""Model and generation-state wrappers over the C ABI (ifr_model / ifr_state)."""
import ctypes

import numpy as np

from ._lib import check, load


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "hidden", "n_layers", "n_head", "n_kv_head", "head_dim", "rotary_dim", "ffn", "vocab",
        "ssm_heads", "ssm_head_dim", "conv_kernel", "context_length", "n_attention_layers", "has_mtp")] + [
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float), ("weight_bytes", ctypes.c_int64)]


class Comm:
    """Tensor-parallel communicator of one rank (NCCL, bound at run time).
    unique_id() on rank 0; every rank passes the same bytes."""

    ID_BYTES = 128

    @staticmethod
    def available():
        return bool(load().ifr_comm_available())

    @staticmethod
    def unique_id():
        buf = (ctypes.c_uint8 * Comm.ID_BYTES)()
        check(load().ifr_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, ctx, rank, world, uid=None):
        self.ctx = ctx
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        idb = (ctypes.c_uint8 * Comm.ID_BYTES).from_buffer_copy(uid) if uid is not None else None
        check(load().ifr_comm_create(ctx.handle, int(rank), int(world), idb, ctypes.byref(h)))
        self.handle = h

    def free(self):
        if getattr(self, "handle", None):
            load().ifr_comm_destroy(self.handle)
            self.handle = None


class Model:
    """A GGUF model resident on the context's device (load_model_cpu analogue,
    src/LoaderCPU.jl:265-437); with a Comm, this rank's tensor-parallel shard."""

    def __init__(self, ctx, path, comm=None):
        self.ctx = ctx
        self.comm = comm
        h = ctypes.c_void_p()
        if comm is None:
            check(load().ifr_model_load_gguf(ctx.handle, path.encode(), ctypes.byref(h)))
        else:
            check(load().ifr_model_load_gguf_tp(ctx.handle, path.encode(), comm.handle, ctypes.byref(h)))
        self.handle = h
        info = ModelInfo()
        check(load().ifr_model_get_info(self.handle, ctypes.byref(info)))
        self.info = info
        sh = (ctypes.c_int32 * 8)()
        check(load().ifr_model_get_shard(self.handle, sh))
        (self.tp_rank, self.tp_world, self.n_head_local, self.n_kv_local, self.ffn_local, self.ffn_off,
         self.vocab_local, self.vocab_off) = list(sh)

    def free(self):
        if getattr(self, "handle", None):
            load().ifr_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class State:
    """KV caches, SSM states and the emitted-token logs of `batch` sequences
    that advance together (one sequence by default)."""

    def __init__(self, model, max_ctx, batch=1):
        self.model = model
        h = ctypes.c_void_p()
        if batch == 1:
            check(load().ifr_state_create(model.handle, int(max_ctx), ctypes.byref(h)))
        else:
            check(load().ifr_state_create_batch(model.handle, int(max_ctx), int(batch), ctypes.byref(h)))
        self.handle = h
        self.max_ctx = max_ctx
        self.batch = batch

    def free(self):
        if getattr(self, "handle", None):
            load().ifr_state_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def reset(self):
        check(load().ifr_state_reset(self.handle))

    def prefill(self, tokens):
        """tokens [n] (one sequence) or [batch][n]; returns the first greedy token(s)"""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if self.batch == 1 and t.ndim == 1:
            first = ctypes.c_int32()
            check(load().ifr_prefill(self.handle, t.ctypes.data_as(ctypes.c_void_p), len(t), ctypes.byref(first)))
            return first.value
        t = t.reshape(self.batch, -1)
        first = np.empty(self.batch, np.int32)
        check(load().ifr_prefill_batch(self.handle, t.ctypes.data_as(ctypes.c_void_p), t.shape[1],
                                       first.ctypes.data_as(ctypes.c_void_p)))
        return first

    def spec_step(self, gamma, drafts=None):
        """asynchronous: MTP draft (or given drafts) -> verify -> accept -> commit"""
        d = None
        if drafts is not None:
            d = np.ascontiguousarray(drafts, dtype=np.int32)
            assert d.size == gamma * self.batch
        check(load().ifr_spec_step(self.handle, int(gamma), d.ctypes.data_as(ctypes.c_void_p) if d is not None else None))

    def spec_step_draft(self, draft, gamma):
        """asynchronous: `draft` (a State of an attention-only draft model on the
        same context) decodes gamma tokens -> verify -> accept -> commit"""
        check(load().ifr_spec_step_draft(self.handle, draft.handle, int(gamma)))

    def draft_mtp(self, gamma):
        """greedy MTP drafts [batch][gamma] (synchronizes)"""
        d = np.empty((self.batch, gamma), np.int32)
        check(load().ifr_draft_mtp(self.handle, int(gamma), d.ctypes.data_as(ctypes.c_void_p)))
        return d

    def verify_step(self, gamma, drafts=None, logits_out=None):
        """target forward over [last, drafts]; logits_out: a device tensor of
        batch * (gamma + 1) * vocab f32 (torch), or None"""
        d = None
        if drafts is not None:
            d = np.ascontiguousarray(drafts, dtype=np.int32)
            assert d.size == gamma * self.batch
        check(load().ifr_verify_step(self.handle, int(gamma), d.ctypes.data_as(ctypes.c_void_p) if d is not None else None,
                                     ctypes.c_void_p(logits_out.data_ptr()) if logits_out is not None else None))

    def rollback(self, accept_count, tokens):
        """commit accept_count[b] drafts + the emitted token of each request"""
        a = np.ascontiguousarray(accept_count, dtype=np.int32).reshape(self.batch)
        t = np.ascontiguousarray(tokens, dtype=np.int32).reshape(self.batch, -1)
        check(load().ifr_rollback(self.handle, a.ctypes.data_as(ctypes.c_void_p), t.ctypes.data_as(ctypes.c_void_p)))

    def capture_draft(self, draft, gamma, steps):
        check(load().ifr_spec_graph_draft(self.handle, draft.handle, int(gamma), int(steps)))

    def capture(self, gamma, steps):
        """capture `steps` MTP spec steps into a CUDA graph (context stream must be capturable)"""
        check(load().ifr_spec_graph(self.handle, int(gamma), int(steps)))

    def launch(self):
        check(load().ifr_spec_graph_launch(self.handle))

    def profile(self, enable=True):
        check(load().ifr_state_profile(self.handle, 1 if enable else 0))

    CATEGORIES = ("lm_head", "draft_lm_head", "layer_gemv", "draft_gemv", "ssm", "attention", "allreduce",
                  "fused_layers")

    def profile_read(self):
        ms = (ctypes.c_double * 8)()
        by = (ctypes.c_int64 * 8)()
        ct = (ctypes.c_int * 8)()
        nl = ctypes.c_int64()
        check(load().ifr_state_profile_read(self.handle, ms, by, ct, ctypes.byref(nl)))
        out = {c: dict(ms=ms[i], bytes=by[i], count=ct[i]) for i, c in enumerate(self.CATEGORIES)}
        return out, nl.value

    FUSED_KINDS = {1: "projection", 2: "ssm", 3: "attn_slices", 4: "attn_combine", 5: "ssm_final"}

    def fused_trace(self, max_phases=1024):
        """[(phase kind, total, fragments, tiles, epilogue, barrier, slowest CTA)]
        in us of the last fused layer-stack launch traced while profiling
        (empty when none); total = from the phase's start to the next's"""
        kinds = (ctypes.c_int * max_phases)()
        us = (ctypes.c_double * (6 * max_phases))()
        n = ctypes.c_int()
        check(load().ifr_state_fused_trace(self.handle, max_phases, kinds, us, ctypes.byref(n)))
        k = n.value
        self.fused_barriers = [tuple(us[6 * k + 4 * i:6 * k + 4 * i + 4]) for i in range(k)] if max_phases >= 2 * k else []
        return [(self.FUSED_KINDS.get(kinds[i], str(kinds[i])),) + tuple(us[6 * i:6 * i + 6]) for i in range(k)]

    def gemv_pass(self, ncols):
        """enqueue the verify's dequant-GEMV launches alone (scratch activations)"""
        check(load().ifr_gemv_pass(self.handle, int(ncols)))

    def read(self, b=0):
        """(emitted tokens, position, last accept count, steps) of request b"""
        n = ctypes.c_int()
        sc = (ctypes.c_int32 * 4)()
        buf = np.empty(self.max_ctx + 16, dtype=np.int32)
        check(load().ifr_state_read_request(self.handle, int(b), buf.ctypes.data_as(ctypes.c_void_p), len(buf),
                                            ctypes.byref(n), sc))
        return buf[:n.value].copy(), sc[0], sc[1], sc[2]

    def last_verify(self):
        """(logits [batch * n][vocab], hidden [batch * n][hidden], tokens [batch * n])
        of the last forward, request-major"""
        info = self.model.info
        n = ctypes.c_int()
        check(load().ifr_state_last_verify(self.handle, None, None, None, ctypes.byref(n)))
        rows = n.value * self.batch
        lg = np.empty((rows, self.model.vocab_local), np.float32)
        hd = np.empty((rows, info.hidden), np.float32)
        tk = np.empty(rows, np.int32)
        check(load().ifr_state_last_verify(self.handle, lg.ctypes.data_as(ctypes.c_void_p),
                                           hd.ctypes.data_as(ctypes.c_void_p),
                                           tk.ctypes.data_as(ctypes.c_void_p), ctypes.byref(n)))
        return lg, hd, tk
