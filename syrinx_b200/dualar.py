"""Host-side mirror of the reference's dual-AR backend interface over the C ABI.

`B200DualAr` carries the method set of the reference trait `DualArBackend`
(crates/syrinx-fish/src/common/dualar.rs:65-136) with the same argument meaning and
error behaviour (a failed call raises, as a `candle_core::Error::Msg` would):
`config`, `reset`, `prefill`, `slow_step`, `first_code`, `fast_expand`, `is_stop` and the
batch variants. `drive` / `drive_batch` are the reference driver loops (dualar.rs:161-364)
written over that interface; `Sampler` is the reference's seeded sampler
(common/sampling.rs). Every tensor op runs in libsyrinx_b200.so on the GPU.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import math

import numpy as np

from . import _lib
from .configs import SX_DTYPE_F32, SX_DTYPE_Q8_0, ModelConfig, SxSamplingParams


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def synth_blob(cfg: ModelConfig, wtype: int = SX_DTYPE_Q8_0, seed: int = 0) -> np.ndarray:
    """Seeded synthetic weights for `cfg` as an SXW1 blob (host memory, uint8)."""
    L = _lib.lib()
    desc = cfg.to_c()
    size = C.c_size_t()
    _lib.check(L.sx_synth_blob_size(C.byref(desc), wtype, C.byref(size)))
    buf = np.empty(size.value, dtype=np.uint8)
    _lib.check(L.sx_synth_blob_write(C.byref(desc), wtype, seed, buf.ctypes.data, size.value))
    return buf


TP_HANDLE_BYTES = 128  # SX_TP_HANDLE_BYTES


class Model:
    """Weights resident on one GPU (replaces `S2Pro::load_with_dtype`, s2/mod.rs:119-167)."""

    def __init__(self, cfg: ModelConfig, blob: np.ndarray, device: int = 0, tp_rank: int = 0, tp_size: int = 1):
        """tp_size > 1: this process holds rank tp_rank's tensor-parallel shard (one process
        per GPU; see syrinx_b200.tp)."""
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self._desc = cfg.to_c()
        self.handle = C.c_void_p()
        if tp_size == 1:
            _lib.check(_lib.lib().sx_model_create(C.byref(self._desc), blob.ctypes.data, blob.nbytes,
                                                  device, C.byref(self.handle)))
        else:
            _lib.check(_lib.lib().sx_model_create_tp(C.byref(self._desc), blob.ctypes.data, blob.nbytes,
                                                     device, tp_rank, tp_size, C.byref(self.handle)))

    def weight_bytes(self) -> int:
        n = C.c_size_t()
        _lib.check(_lib.lib().sx_model_weight_bytes(self.handle, C.byref(n)))
        return n.value

    def close(self):
        if self.handle:
            _lib.lib().sx_model_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclasses.dataclass
class SlowStep:
    """`SlowStep` (dualar.rs:44-51): raw unmasked logits [vocab] and the fast-AR hidden."""
    semantic_logits: np.ndarray
    hidden: np.ndarray


class B200DualAr:
    """`DualArBackend` over the B200 kernels, one session of up to `max_batch` sequences."""

    def __init__(self, model: Model, max_ctx: int, max_batch: int = 1, kv_dtype: int = SX_DTYPE_F32):
        """kv_dtype SX_DTYPE_F32 (default, the reference CPU cache: token-exact greedy output)
        or SX_DTYPE_BF16 (half the KV bytes, for long contexts and batched decode)."""
        self.model = model
        self.cfg = model.cfg
        self.max_ctx = max_ctx
        self.max_batch = max_batch
        self.kv_dtype = kv_dtype
        self.handle = C.c_void_p()
        _lib.check(_lib.lib().sx_session_create_ex(model.handle, max_batch, max_ctx, kv_dtype,
                                                   C.byref(self.handle)))

    # -- tensor parallelism ----------------------------------------------------------------
    def tp_handle(self) -> bytes:
        """This rank's exchange handle (SX_TP_HANDLE_BYTES bytes) for the other ranks."""
        buf = (C.c_uint8 * TP_HANDLE_BYTES)()
        _lib.check(_lib.lib().sx_session_tp_handle(self.handle, buf))
        return bytes(buf)

    def tp_connect(self, handles: list[bytes]) -> None:
        """Map every rank's exchange region; `handles` in rank order, this rank's included."""
        blob = b"".join(handles)
        if len(blob) != TP_HANDLE_BYTES * len(handles):
            raise ValueError("tensor-parallel handles must be SX_TP_HANDLE_BYTES each")
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _lib.check(_lib.lib().sx_session_tp_connect(self.handle, buf))

    def fill_kv_synthetic(self, length: int, seed: int, seq: int = 0) -> None:
        """Benchmark surface: an empty sequence gets `length` positions of seeded KV values
        (as if prefilled); a later prefill appends after them."""
        _lib.check(_lib.lib().sx_session_fill_kv_synthetic(self.handle, seq, length, seed))

    def tp_set_timeout(self, timeout_ns: int) -> None:
        """Longest wait of a residual exchange for a peer (ns); before the first decode loop."""
        _lib.check(_lib.lib().sx_session_tp_set_timeout(self.handle, int(timeout_ns)))

    def tp_disconnect(self) -> None:
        """Unmap the peers (every rank, before any rank closes its session)."""
        _lib.check(_lib.lib().sx_session_tp_disconnect(self.handle))

    # -- DualArBackend ------------------------------------------------------------------
    def config(self) -> ModelConfig:
        return self.cfg

    def reset(self, max_seq_len: int | None = None) -> None:
        if max_seq_len is not None and max_seq_len > self.max_ctx:
            raise _lib.SyrinxError(-7, "max_seq_len exceeds the session capacity")
        _lib.check(_lib.lib().sx_session_reset(self.handle))

    def _outs(self, n: int = 1):
        logits = np.empty((n, self.cfg.vocab_size), np.float32)
        hidden = np.empty((n, self.cfg.slow.dim), np.float32)
        return logits, hidden

    def prefill(self, prompt: np.ndarray) -> SlowStep:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        if p.ndim == 1:
            p = p[None, :]
        assert p.shape[0] == self.cfg.frame_width, "prompt must be [1 + num_codebooks, T]"
        logits, hidden = self._outs()
        _lib.check(_lib.lib().sx_prefill(self.handle, _p(p, C.c_uint32), p.shape[1],
                                         _p(logits, C.c_float), _p(hidden, C.c_float)))
        return SlowStep(logits[0], hidden[0])

    def slow_step(self, frame, pos: int) -> SlowStep:
        f = np.ascontiguousarray(frame, dtype=np.uint32).reshape(-1)
        assert f.size == self.cfg.frame_width, "frame must be [1 + num_codebooks]"
        logits, hidden = self._outs()
        _lib.check(_lib.lib().sx_slow_step(self.handle, _p(f, C.c_uint32), pos,
                                           _p(logits, C.c_float), _p(hidden, C.c_float)))
        return SlowStep(logits[0], hidden[0])

    def first_code(self, semantic_token: int) -> int:
        return int(_lib.lib().sx_first_code(self.model.handle, semantic_token))

    def fast_expand(self, hidden, first_code: int, sampler: "Sampler") -> list[int]:
        """Fast AR conditioned on the hidden of the last slow step of this session
        (`hidden` is accepted for signature parity; the device keeps its own copy)."""
        codes = np.empty(self.cfg.num_codebooks, np.uint32)

        def _cb(_user, logits_ptr, n):
            logits = np.ctypeslib.as_array(logits_ptr, shape=(n,)).copy()
            return sampler.sample_codebook(logits, [])

        fn = _lib.SAMPLE_FN(_cb)
        _lib.check(_lib.lib().sx_fast_expand(self.handle, first_code, fn, None, _p(codes, C.c_uint32)))
        return [int(c) for c in codes]

    def fast_expand_greedy(self, first_code: int) -> list[int]:
        codes = np.empty(self.cfg.num_codebooks, np.uint32)
        _lib.check(_lib.lib().sx_fast_expand_greedy(self.handle, first_code, _p(codes, C.c_uint32)))
        return [int(c) for c in codes]

    def is_stop(self, semantic_token: int) -> bool:
        return semantic_token in self.cfg.stop_ids()

    # -- batched ------------------------------------------------------------------------
    def prefill_batch(self, prompts: list[np.ndarray]) -> SlowStep:
        ps = [np.ascontiguousarray(p, dtype=np.uint32) for p in prompts]
        lens = np.array([p.shape[1] for p in ps], np.int32)
        flat = np.concatenate([p.reshape(-1) for p in ps]).astype(np.uint32)
        logits, hidden = self._outs(len(ps))
        _lib.check(_lib.lib().sx_prefill_batch(self.handle, _p(flat, C.c_uint32), _p(lens, C.c_int32), len(ps),
                                               _p(logits, C.c_float), _p(hidden, C.c_float)))
        return SlowStep(logits, hidden)

    def slow_step_batch(self, frames: list[list[int]], active: list[bool] | None = None) -> SlowStep:
        f = np.ascontiguousarray(frames, dtype=np.uint32)
        n = f.shape[0]
        act = np.array([1] * n if active is None else [int(a) for a in active], np.uint8)
        logits, hidden = self._outs(n)
        _lib.check(_lib.lib().sx_slow_step_batch(self.handle, _p(f, C.c_uint32), _p(act, C.c_uint8), n,
                                                 _p(logits, C.c_float), _p(hidden, C.c_float)))
        return SlowStep(logits, hidden)

    def fast_expand_batch_greedy(self, first_codes: list[int], active: list[bool] | None = None) -> np.ndarray:
        n = len(first_codes)
        fc = np.array(first_codes, np.uint32)
        act = np.array([1] * n if active is None else [int(a) for a in active], np.uint8)
        out = np.empty((n, self.cfg.num_codebooks), np.uint32)
        _lib.check(_lib.lib().sx_fast_expand_batch_greedy(self.handle, _p(fc, C.c_uint32), _p(act, C.c_uint8), n,
                                                          _p(out, C.c_uint32)))
        return out

    # -- device-resident greedy loops -----------------------------------------------------
    def frame_step_greedy(self, frame_in, mask_stop: bool = False):
        out = np.empty(self.cfg.frame_width, np.uint32)
        stopped = C.c_int32()
        fin = None if frame_in is None else np.ascontiguousarray(frame_in, dtype=np.uint32)
        _lib.check(_lib.lib().sx_frame_step_greedy(self.handle, None if fin is None else _p(fin, C.c_uint32),
                                                   int(mask_stop), _p(out, C.c_uint32), C.byref(stopped)))
        return out, bool(stopped.value)

    def decode_greedy(self, n_frames: int, mask_stop: bool = False) -> np.ndarray:
        out = np.zeros((n_frames, self.cfg.frame_width), np.uint32)
        n = C.c_int32()
        _lib.check(_lib.lib().sx_decode_greedy(self.handle, n_frames, int(mask_stop), _p(out, C.c_uint32),
                                               C.byref(n)))
        return out[: n.value]

    def decode_sample(self, n_frames: int, seed: int, sampling: "SamplingParams") -> np.ndarray:
        """Device-sampled frames of sequence 0 after prefill ([frames, 1 + C]); the same draws
        as the reference drive loop with Sampler(seed, sampling)."""
        out = np.zeros((n_frames, self.cfg.frame_width), np.uint32)
        n = C.c_int32()
        params = sampling.to_c()
        _lib.check(_lib.lib().sx_decode_sample(self.handle, n_frames, seed & 0xFFFFFFFFFFFFFFFF, C.byref(params),
                                               _p(out, C.c_uint32), C.byref(n)))
        return out[: n.value]

    def decode_greedy_batch(self, n: int, n_frames: int, mask_stop: bool = False) -> list[np.ndarray]:
        out = np.zeros((n, n_frames, self.cfg.frame_width), np.uint32)
        counts = np.zeros(n, np.int32)
        _lib.check(_lib.lib().sx_decode_greedy_batch(self.handle, n, n_frames, int(mask_stop), _p(out, C.c_uint32),
                                                     _p(counts, C.c_int32)))
        return [out[i, : counts[i]] for i in range(n)]

    def lm_step_tokens(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        _lib.check(_lib.lib().sx_lm_step_tokens(self.handle, _p(t, C.c_uint32), t.size, _p(logits, C.c_float)))
        return logits

    def lm_step_embeds(self, embeds: np.ndarray) -> np.ndarray:
        """`Qwen2Lm::step_logits_cached(embeds)`: [t_new, dim] input embeddings through the
        cached forward; the last position's logits."""
        e = np.ascontiguousarray(embeds, dtype=np.float32).reshape(-1, self.cfg.slow.dim)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        _lib.check(_lib.lib().sx_lm_step_embeds(self.handle, _p(e, C.c_float), e.shape[0], _p(logits, C.c_float)))
        return logits

    def set_stream(self, cuda_stream: int | None) -> None:
        """Enqueue device work on an external cudaStream_t (an int handle), or None."""
        _lib.check(_lib.lib().sx_session_set_stream(self.handle, C.c_void_p(cuda_stream or 0)))

    def profile_gemv(self, kind: int, n_launches: int) -> None:
        _lib.check(_lib.lib().sx_profile_gemv(self.handle, kind, n_launches))

    def profile_stack(self, fast: bool = False) -> dict:
        """Phase timing of one persistent-stack launch (us): total, per-layer mean of each
        phase, the final phase and the setup."""
        out = np.zeros(28, np.float32)
        _lib.check(_lib.lib().sx_profile_stack(self.handle, int(fast), _p(out, C.c_float)))
        r = {"total": float(out[0]), "setup": float(out[1]), "final": float(out[2])}
        for p, name in enumerate(["wqkv", "attention", "wo", "w13", "w2"]):
            r[name] = {k: round(float(out[3 + 4 * p + i]), 2)
                       for i, k in enumerate(["phase", "prologue", "arrival", "barrier"])}
        r["attention_cta0"] = {k: round(float(out[23 + i]), 2) for i, k in enumerate(
            ["merge_loads", "scale", "norm_rope_append", "key_loop", "write"])}
        return r

    def seq_len(self, seq: int = 0) -> int:
        v = C.c_int32()
        _lib.check(_lib.lib().sx_session_len(self.handle, seq, C.byref(v)))
        return v.value

    def close(self):
        if self.handle:
            _lib.lib().sx_session_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- the reference sampler (common/sampling.rs) ---------------------------------------------

@dataclasses.dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 0.9
    top_k: int = 30
    repetition_penalty: float = 1.1
    ras_win_size: int = 10
    ras_high_temp: float = 1.0
    ras_high_top_p: float = 0.9

    def to_c(self) -> SxSamplingParams:
        return SxSamplingParams(self.temperature, self.top_p, self.top_k, self.repetition_penalty,
                                self.ras_win_size, self.ras_high_temp, self.ras_high_top_p)


GREEDY = SamplingParams(top_k=1)


class SplitMix64:
    def __init__(self, seed: int):
        self.state = seed & 0xFFFFFFFFFFFFFFFF

    def next_u64(self) -> int:
        M = 0xFFFFFFFFFFFFFFFF
        self.state = (self.state + 0x9E3779B97F4A7C15) & M
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) * (1.0 / (1 << 53))


def logits_to_probs(logits: np.ndarray, temperature: float, top_p: float, top_k: int) -> np.ndarray:
    """Nucleus recipe of sampling.rs:189-245 (sort desc, ties by index; keep top-1)."""
    logits = np.asarray(logits, np.float32)
    n = logits.size
    order = sorted(range(n), key=lambda i: (-float(logits[i]) if not math.isnan(logits[i]) else 0.0, i))
    mx = logits[order[0]] if n else np.float32(0)
    exps = [math.exp(float(np.float32(logits[i] - mx))) for i in order]
    total = sum(exps)
    k_cap = n if top_k == 0 else top_k
    keep = np.zeros(n, bool)
    cum = 0.0
    for rank, i in enumerate(order):
        if rank == 0 or (cum <= float(np.float32(top_p)) and rank < k_cap):
            keep[i] = True
        else:
            break
        cum += exps[rank] / total
    t = np.float32(max(temperature, 1e-5))
    scaled = (logits / t).astype(np.float32)
    kept_max = max(float(scaled[i]) for i in range(n) if keep[i])
    probs = np.zeros(n, np.float32)
    psum = 0.0
    for i in range(n):
        if keep[i]:
            e = math.exp(float(np.float32(scaled[i] - np.float32(kept_max))))
            probs[i] = np.float32(e)
            psum += e
    if psum > 0:
        probs = np.array([np.float32(float(p) / psum) for p in probs], np.float32)
    return probs


def multinomial1(probs: np.ndarray, rng: SplitMix64) -> int:
    total = float(sum(float(p) for p in probs))
    if total <= 0.0:
        return 0
    u = rng.next_f64() * total
    acc = 0.0
    for i, p in enumerate(probs):
        acc += float(p)
        if u < acc:
            return i
    return len(probs) - 1


class Sampler:
    """`Sampler` (sampling.rs:110-168): one PRNG stream shared by slow and fast draws."""

    def __init__(self, seed: int, params: SamplingParams):
        self.rng = SplitMix64(seed)
        self.params = params

    def sample_codebook(self, logits: np.ndarray, recent) -> int:
        p = self.params
        work = np.array(logits, np.float32)
        if abs(p.repetition_penalty - 1.0) >= np.finfo(np.float32).eps:
            for i in recent:
                if i < work.size:
                    work[i] = work[i] / p.repetition_penalty if work[i] > 0 else work[i] * p.repetition_penalty
        return multinomial1(logits_to_probs(work, p.temperature, p.top_p, p.top_k), self.rng)

    def sample_semantic(self, logits: np.ndarray, window, cfg: ModelConfig) -> int:
        p = self.params
        c = np.array(logits, np.float32)
        allowed = np.zeros(c.size, bool)
        allowed[cfg.semantic_begin_id: cfg.semantic_end_id + 1] = True
        for s in cfg.stop_ids():
            allowed[s] = True
        c[~allowed] = -np.inf
        normal = multinomial1(logits_to_probs(c, p.temperature, p.top_p, p.top_k), self.rng)
        high = multinomial1(logits_to_probs(c, p.ras_high_temp, p.ras_high_top_p, p.top_k), self.rng)
        sem = cfg.semantic_begin_id <= normal <= cfg.semantic_end_id
        return high if (normal in window and sem) else normal


def drive(backend: B200DualAr, prompt: np.ndarray, max_new_frames: int, seed: int,
          sampling: SamplingParams) -> np.ndarray:
    """The reference `drive` loop (dualar.rs:161-230); returns the [num_codebooks, T] codes."""
    cfg = backend.config()
    backend.reset(backend.max_ctx)
    sampler = Sampler(seed, sampling)
    prompt = np.asarray(prompt)
    frames, window = [], []
    ras_win = max(sampling.ras_win_size, 1)
    step = backend.prefill(prompt)
    pos = prompt.shape[-1]
    while True:
        semantic = sampler.sample_semantic(step.semantic_logits, window, cfg)
        if backend.is_stop(semantic):
            break
        first = backend.first_code(semantic)
        frame = backend.fast_expand(step.hidden, first, sampler)
        frames.append(frame)
        window.append(semantic)
        if len(window) > ras_win:
            window.pop(0)
        if len(frames) >= max_new_frames:
            break
        if pos + 1 >= backend.max_ctx:
            break
        step = backend.slow_step([semantic] + frame, pos)
        pos += 1
    return np.array(frames, np.uint32).reshape(len(frames), cfg.num_codebooks).T.copy()
