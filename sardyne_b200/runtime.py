"""Model / Context / generate over the engine C-ABI — the reference's runtime interface
(reference sardyne/runtime.py:34-140: same classes, arguments, return values and errors).

``lib`` defaults to this package's libsardyne.so; any library exporting the reference's engine_*
symbols with the reference's signatures works the same way.
"""
import ctypes

import numpy as np

from . import capi


NCCL_ID_BYTES = 128


def set_shard(rank: int, world: int, nccl_id: bytes | None = None) -> None:
    """Configure the next Model load of this process as rank `rank` of `world` (one GPU per process;
    world 1 = unsharded). Sharded ranks keep attention and the router, split the FFN rows, the
    experts and the vocabulary, and all return the one-GPU logits. Every rank must then load the
    same model and run the same eval calls."""
    lib = capi.lib()
    buf = (ctypes.c_char * NCCL_ID_BYTES).from_buffer_copy(nccl_id) if nccl_id else None
    if lib.sdy_engine_set_shard(rank, world, buf) != 0:
        raise ValueError(capi.last_error())


def new_nccl_id() -> bytes:
    buf = (ctypes.c_char * NCCL_ID_BYTES)()
    if capi.lib().sdy_nccl_unique_id(buf) != 0:
        raise RuntimeError(capi.last_error())
    return bytes(buf)


def shard_from_torch(group=None) -> tuple[int, int]:
    """set_shard from a torch.distributed process group: rank 0 creates the NCCL id and
    broadcasts it. Returns (rank, world)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nccl_id = None
    if world > 1:
        obj = [new_nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        nccl_id = obj[0]
    set_shard(rank, world, nccl_id)
    return rank, world


class Model:
    def __init__(self, path, lib=None):
        self._lib = lib or capi.lib()
        self._h = None
        err = ctypes.create_string_buffer(512)
        self._h = self._lib.engine_model_load(str(path).encode(), err, len(err))
        if not self._h:
            raise ValueError(err.value.decode("utf-8", errors="replace"))
        self.info = capi.EngineModelInfo()
        self._lib.engine_model_get_info(self._h, ctypes.byref(self.info))
        self.path = path

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.engine_model_free(self._h)
            self._h = None


class Context:
    def __init__(self, model: Model, max_seq: int = 2048, n_batch: int = 64, logits_all: bool = False,
                 n_threads: int = 0):
        self.model = model
        self._lib = model._lib
        self._h = None
        self.max_seq = min(max_seq, model.info.max_pos)
        self.n_batch = n_batch
        self.logits_all = logits_all
        err = ctypes.create_string_buffer(512)
        self._h = self._lib.engine_ctx_new(model._h, self.max_seq, n_batch, int(logits_all), n_threads, err, len(err))
        if not self._h:
            raise ValueError(err.value.decode("utf-8", errors="replace"))
        self.n_threads = self._lib.engine_ctx_n_threads(self._h)

    def __del__(self):
        if getattr(self, "_h", None):
            self._lib.engine_ctx_free(self._h)
            self._h = None

    @property
    def n_past(self) -> int:
        return self._lib.engine_n_past(self._h)

    def reset(self):
        self._lib.engine_reset(self._h)

    def truncate(self, n: int):
        if self._lib.engine_truncate(self._h, n) != 0:
            raise ValueError(self._lib.engine_last_error(self._h).decode("utf-8", errors="replace"))

    def eval(self, tokens) -> np.ndarray:
        """Logits (a copy): [n_tokens, vocab] with logits_all, else [vocab] of the last token."""
        tokens = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).reshape(-1))
        if tokens.size == 0:
            raise ValueError("nessun token in ingresso")
        if tokens.min() < np.iinfo(np.int32).min or tokens.max() > np.iinfo(np.int32).max:
            raise ValueError("id di token fuori dall'intervallo int32")
        tokens = tokens.astype(np.int32)
        step = self.n_batch if self.logits_all else tokens.size
        outs = []
        for i in range(0, tokens.size, step):
            part = tokens[i:i + step]
            p = part.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
            if self._lib.engine_eval(self._h, p, part.size) != 0:
                raise ValueError(self._lib.engine_last_error(self._h).decode("utf-8", errors="replace"))
            n = self._lib.engine_n_logits(self._h)
            outs.append(np.ctypeslib.as_array(self._lib.engine_logits(self._h), shape=(n, self.model.info.n_vocab)).copy())
        out = np.concatenate(outs)
        return out if self.logits_all else out[-1]


def generate(ctx: Context, prompt, n_new: int, eos_ids=(), on_token=None, sampler=None) -> list[int]:
    """Prefill the prompt, then one token at a time (greedy unless a sampler is given)."""
    eos_ids = {eos_ids} if isinstance(eos_ids, int) else set(eos_ids)
    pick = sampler or (lambda logits, history: int(np.argmax(logits)))
    history, out = list(prompt), []
    if n_new <= 0:
        return out
    ctx.reset()
    logits = ctx.eval(prompt)
    if ctx.logits_all:
        logits = logits[-1]
    for _ in range(n_new):
        nxt = pick(logits, history)
        history.append(nxt)
        out.append(nxt)
        if on_token:
            on_token(nxt)
        if nxt in eos_ids or ctx.n_past >= ctx.max_seq:
            break
        logits = ctx.eval([nxt])
        if ctx.logits_all:
            logits = logits[-1]
    return out
