"""Host-side mirror of the reference's graft interface over the C ABI.

Names follow the reference (Hinedes/GLT): ``GraftConfig`` carries the fields
of src/config.hpp:40-91 with the same defaults, ``GraftModel`` owns what the
reference splits between ModelWeights, VramArena and GraftWeights
(src/types.hpp:127-201), and its methods map to forward_model / the training
loop (grafting.hip:224-271, 954-1172).  Every call goes through
libglt_b200.so; tensors are torch CUDA tensors used as plain device memory.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, fields

import torch

from . import _lib
from ._lib import GLT_OK, GltModelConfig, GltStepStats, GltEvalStats, check, lib

LAYOUT_OVERLAY, LAYOUT_CONCAT = 0, 1
MODEL_DECODER, MODEL_MLP_BLOCK = 0, 1
W_EMBED, W_LM_HEAD, W_FINAL_NORM, W_IN_NORM, W_Q, W_K, W_V, W_O, W_POST_NORM, W_GATE, W_UP, W_DOWN = range(12)
# per-kind kernel timing slots (GLT_PROF_* in include/glt_graft.h)
PROF_NAMES = ["gate_up_fwd", "down_fwd", "delta_down", "qkv", "o_proj", "attn_fwd", "dh",
              "recompute_swiglu_bwd", "wgrad_down", "wgrad_gate_up", "dx_gate_up", "do",
              "attn_bwd", "dx_qkv", "lm_head", "lm_dx", "cross_entropy", "delta_expand",
              "graft_dgrad", "rmsnorm", "rope", "adamw"]
PROF_KINDS = len(PROF_NAMES)


@dataclass
class GraftConfig:
    """src/config.hpp:40-91 (+ the CLI-level lr / layout / tie flag)."""
    hidden_dim: int = 2048
    intermediate_dim: int = 11008
    slice_dim: int = 2752
    vocab_size: int = 128256
    num_layers: int = 36
    num_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 0
    max_domains: int = 4
    domain_id: int = 0
    layout: int = LAYOUT_OVERLAY
    tie_embeddings: int = 1
    rms_norm_eps: float = 1e-6
    lm_loss_scale: float = 1.0
    lambda_silence: float = 5.0
    rope_theta: float = 5000000.0
    graft_layer_start: int = 0
    graft_layer_end: int = 35
    graft_proj_gate: int = 0
    graft_proj_up: int = 0
    graft_proj_down: int = 1
    allow_expansion_trap: int = 0
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_eps: float = 1e-8
    adam_weight_decay: float = 0.01
    gradient_clip_norm: float = 1.0
    lr_warmup_steps: int = 20
    lr_peak: float = 2e-4
    no_rope_layers: list = field(default_factory=list)

    def to_c(self) -> GltModelConfig:
        c = GltModelConfig()
        for f in fields(self):
            if f.name == "no_rope_layers":
                continue
            setattr(c, f.name, getattr(self, f.name))
        c.no_rope_mask_len = len(self.no_rope_layers)
        for i, v in enumerate(self.no_rope_layers):
            c.no_rope_mask[i] = int(v)
        return c

    def validate(self, batch_size: int, mode: int = 0) -> None:
        check(lib.glt_config_validate(C.byref(self.to_c()), batch_size, mode))

    def get_lr(self, step: int, total_steps: int) -> float:
        return float(lib.glt_get_lr(C.byref(self.to_c()), step, total_steps))

    @property
    def h_slice_dim(self) -> int:
        return self.hidden_dim if self.layout == LAYOUT_CONCAT else self.hidden_dim // self.max_domains


def default_config() -> GraftConfig:
    c = GltModelConfig()
    check(lib.glt_config_default(C.byref(c)))
    kw = {f.name: getattr(c, f.name) for f in fields(GraftConfig) if f.name != "no_rope_layers"}
    return GraftConfig(**kw)


def _stream(stream=None) -> C.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def memcpy(dst: int, src: int, nbytes: int, sync: bool = True, stream=None) -> None:
    check(lib.glt_memcpy(C.c_void_p(dst), C.c_void_p(src), nbytes, _stream(stream), int(sync)))


class GraftModel:
    """Frozen bf16 base + fp32 graft on the current CUDA device."""

    def __init__(self, cfg: GraftConfig, batch_size: int, seq_len: int, kind: int = MODEL_DECODER):
        self.cfg = cfg
        self.B, self.T = batch_size, seq_len
        self._c = cfg.to_c()
        h = C.c_void_p()
        check(lib.glt_model_create(C.byref(self._c), batch_size, seq_len, kind, C.byref(h)))
        self.handle = h
        self.kind = kind

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib.glt_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    # --- weights --------------------------------------------------------------
    def init_random(self, seed: int = 0, std: float = 0.02, graft_std: float = 0.02,
                    graft_down_std: float = 0.0) -> None:
        check(lib.glt_model_init_random(self.handle, seed, std, graft_std, graft_down_std))

    def set_weight(self, layer: int, which: int, t: torch.Tensor) -> None:
        t = t.detach().to(device="cuda", dtype=torch.bfloat16).contiguous()
        check(lib.glt_model_set_weight(self.handle, layer, which, C.c_void_p(t.data_ptr()),
                                       t.numel(), 0, _stream()))
        torch.cuda.current_stream().synchronize()

    def graft_pointers(self):
        w, g, m, v = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
        n = C.c_int64()
        check(lib.glt_model_graft_buffers(self.handle, C.byref(w), C.byref(g), C.byref(m),
                                          C.byref(v), C.byref(n)))
        return dict(weight=w.value, grad=g.value, adam_m=m.value, adam_v=v.value), n.value

    def read_graft(self, which: str = "weight") -> torch.Tensor:
        ptrs, n = self.graft_pointers()
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        memcpy(out.data_ptr(), ptrs[which], n * 4)
        return out

    def write_graft(self, which: str, t: torch.Tensor) -> None:
        ptrs, n = self.graft_pointers()
        t = t.detach().to(device="cuda", dtype=torch.float32).contiguous()
        assert t.numel() == n
        memcpy(ptrs[which], t.data_ptr(), n * 4)
        if which == "weight":
            check(lib.glt_model_refresh_graft(self.handle, _stream()))
            torch.cuda.current_stream().synchronize()

    def activation(self, which: int, layer: int, dtype=torch.bfloat16) -> torch.Tensor:
        p, n = C.c_void_p(), C.c_int64()
        check(lib.glt_model_activation(self.handle, which, layer, C.byref(p), C.byref(n)))
        out = torch.empty(n.value, dtype=dtype, device="cuda")
        memcpy(out.data_ptr(), p.value, n.value * out.element_size())
        return out

    # --- steps ----------------------------------------------------------------
    def train_step(self, ids: torch.Tensor, ood_mask: torch.Tensor, step: int, total_steps: int,
                   want_stats: bool = True) -> dict | None:
        host = int(ids.device.type == "cpu")
        ids = ids.to(torch.int32).contiguous()
        ood_mask = ood_mask.to(torch.int32).contiguous()
        st = GltStepStats()
        check(lib.glt_train_step(self.handle, C.c_void_p(ids.data_ptr()),
                                 C.c_void_p(ood_mask.data_ptr()), host, step, total_steps,
                                 C.byref(st) if want_stats else None, _stream()))
        if not want_stats:
            return None
        return {f: getattr(st, f) for f, _ in GltStepStats._fields_}

    def step_stats(self, step: int) -> dict:
        """Stats of an enqueued training step (one of the last two), waiting for that step only."""
        st = GltStepStats()
        check(lib.glt_model_step_stats(self.handle, step, C.byref(st)))
        return {f: getattr(st, f) for f, _ in GltStepStats._fields_}

    def forward(self, ids: torch.Tensor, use_graft: bool = True, want_logits: bool = True):
        host = int(ids.device.type == "cpu")
        ids = ids.to(torch.int32).contiguous()
        logits = None
        if want_logits:
            logits = torch.empty(ids.numel(), self.cfg.vocab_size, dtype=torch.bfloat16, device="cuda")
        check(lib.glt_forward(self.handle, C.c_void_p(ids.data_ptr()), host, int(use_graft),
                              C.c_void_p(logits.data_ptr()) if logits is not None else None,
                              _stream()))
        return logits

    def eval(self, ids: torch.Tensor, use_graft: bool = True) -> dict:
        """Eval-only / shadow-eval metrics over ids [num_sequences, seq_len]
        (grafting.hip:446-713): tokens, mean_ce, ppl, logits_sum, logits_l2,
        logits_hash, graft_forward_calls."""
        host = int(ids.device.type == "cpu")
        ids = ids.to(torch.int32).contiguous()
        st = GltEvalStats()
        check(lib.glt_model_eval(self.handle, C.c_void_p(ids.data_ptr()), ids.shape[0], host,
                                 int(use_graft), C.byref(st), _stream()))
        return {f: getattr(st, f) for f, _ in GltEvalStats._fields_}

    def shadow_bake(self) -> None:
        """Bake the graft into the base weights and free the graft storage."""
        check(lib.glt_model_shadow_bake(self.handle, _stream()))

    def block_step(self, x: torch.Tensor, y: torch.Tensor, lr: float, step: int = 0,
                   outputs: bool = True):
        """MLP-block step; with outputs=False nothing is read back (no host sync)."""
        x = x.to(device="cuda", dtype=torch.bfloat16).contiguous()
        y = y.to(device="cuda", dtype=torch.float32).contiguous()
        if not outputs:
            check(lib.glt_block_step(self.handle, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                     lr, step, None, None, None, _stream()))
            return None
        out = torch.empty_like(x)
        dx = torch.empty(x.shape, dtype=torch.float32, device="cuda")
        loss = C.c_float()
        check(lib.glt_block_step(self.handle, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                 lr, step, C.byref(loss), C.c_void_p(out.data_ptr()),
                                 C.c_void_p(dx.data_ptr()), _stream()))
        return dict(loss=loss.value, out=out, dx=dx)

    def mlp_store(self, mode: int = -1) -> tuple[bool, int]:
        """Stored MLP activations: mode 0 recompute, 1 store, 2 auto, -1 query.
        Returns (active, bytes)."""
        act = C.c_int32()
        nb = C.c_int64()
        check(lib.glt_model_mlp_store(self.handle, int(mode), C.byref(act), C.byref(nb)))
        return bool(act.value), int(nb.value)

    def profile(self, enable: bool) -> None:
        check(lib.glt_model_profile(self.handle, int(enable)))

    def profile_read(self, reset: bool = True) -> tuple[list[float], list[int]]:
        ms = (C.c_double * PROF_KINDS)()
        n = (C.c_int64 * PROF_KINDS)()
        check(lib.glt_model_profile_read(self.handle, ms, n, int(reset)))
        return list(ms), list(n)

    # --- data parallel --------------------------------------------------------
    @staticmethod
    def dp_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib.glt_dp_unique_id(buf, 128))
        return buf.raw

    def dp_init(self, unique_id: bytes, rank: int, world: int) -> None:
        buf = C.create_string_buffer(unique_id, 128)
        check(lib.glt_dp_init(self.handle, buf, rank, world))

    def dp_finalize(self) -> None:
        check(lib.glt_dp_finalize(self.handle))

    def dp_async_error(self) -> int:
        """The communicator's asynchronous NCCL result (0 = ncclSuccess)."""
        r = C.c_int32()
        st = lib.glt_dp_async_error(self.handle, C.byref(r))
        if st != GLT_OK and r.value == 0:
            check(st)
        return r.value

    def dp_abort(self) -> None:
        """Abort the data-parallel communicator without waiting for the other
        ranks (a peer has left); the model then trains on its own GPU."""
        check(lib.glt_dp_abort(self.handle))


class PeerLost(RuntimeError):
    """A data-parallel peer left or stopped posting steps."""

    def __init__(self, peer: int, last_step: int, wanted: int, left: bool):
        what = "left" if left else f"posted step {last_step} and nothing newer"
        super().__init__(f"rank {peer} {what}; step {wanted} was expected")
        self.peer, self.last_step, self.wanted, self.left = peer, last_step, wanted, left


class PeerMonitor:
    """Host-side liveness of the data-parallel ranks, checked between steps.

    The library's all-reduce runs inside the training step; a peer that has
    crashed or left would make the others' next collective wait for it.  Each
    rank posts the index of every step it has finished to the job's key-value
    store (a torch.distributed Store, e.g. a TCPStore); before a rank enqueues
    step k it checks that every peer has finished step k-1, and raises
    PeerLost -- with no collective in flight -- when a peer has posted its
    leave marker or has been silent for `timeout_s`.  The caller then aborts
    the communicator (GraftModel.dp_abort) and exits or trains alone.  The
    reference is single-GPU and has no counterpart."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0, prefix: str = "glt_dp"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def _read(self, key: str) -> int | None:
        return int(self.store.get(key)) if self.store.check([key]) else None

    def beat(self, step: int) -> None:
        """This rank has finished `step`."""
        self.store.set(self._key("step", self.rank), str(int(step)))

    def leave(self) -> None:
        """This rank takes no further steps: peers waiting for a later step raise
        PeerLost at once instead of after the timeout."""
        self.store.set(self._key("left", self.rank), "1")

    def wait_peers(self, step: int) -> None:
        """Return once every peer has finished `step`; raise PeerLost otherwise."""
        import time
        deadline = time.monotonic() + self.timeout_s
        for r in range(self.world):
            if r == self.rank:
                continue
            while True:
                last = self._read(self._key("step", r))
                last = -1 if last is None else last
                if last >= step:
                    break
                if self._read(self._key("left", r)) is not None:
                    raise PeerLost(r, last, step, True)
                if time.monotonic() > deadline:
                    raise PeerLost(r, last, step, False)
                time.sleep(0.005)
