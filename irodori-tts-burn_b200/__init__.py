"""irodori-b200: B200 (sm_100a) engine for Irodori-TTS rectified-flow sampling
and DACVAE decoding.

Host-side mirror of the Irodori-TTS-burn crate's inference API for this path
(src/inference.rs:83-254, src/rf/params.rs:9-247, src/codec/weights.rs:27-33)
over the C ABI in ``include/irodori_b200.h``.  Names, argument meaning and
error behaviour follow the reference:

    engine = (InferenceBuilder(device=0)          # Unconfigured
              .load_weights("model.safetensors")  # -> Loaded
              .with_default_sampling()            # -> Ready
              .build())                           # -> InferenceEngine
    latent = engine.sample(SamplingRequest(text_ids=..., text_mask=..., sequence_length=750, ...))

All compute runs in ``libirodori_b200.so`` on the GPU; there is no CPU path.
Loading the library fails loudly when it has not been built.
"""

from __future__ import annotations

import ctypes
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Optional, Sequence

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libirodori_b200.so"

# irt_status (include/irodori_b200.h) -> IrodoriError variant names (src/error.rs:3-60)
IRT_OK = 0
STATUS_NAMES = {
    1: "Config", 2: "Shape", 3: "MissingInput", 4: "UnsupportedMode", 5: "Io", 6: "Json", 7: "Weight",
    8: "WrongDim", 9: "Dtype", 10: "SafeTensors", 11: "NoConfig", 20: "Cuda", 21: "State", 22: "InvalidArgument",
    23: "OutOfMemory",
}
PREC = {"bf16": 0, "f32": 1}
METHODS = {"euler": 0, "heun": 1, "plms4": 2}
MODES = {"independent": 0, "joint": 1, "alternating": 2}
MEM_HOST, MEM_DEVICE = 0, 1


class IrodoriError(Exception):
    """Error raised by the engine; ``kind`` is the IrodoriError variant name."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = STATUS_NAMES.get(status, f"Status{status}")
        super().__init__(message)


class ConfigError(IrodoriError):
    pass


class StateError(IrodoriError):
    pass


def _error_class(status: int):
    return {1: ConfigError, 21: StateError}.get(status, IrodoriError)


# ---------------------------------------------------------------------------
# C structs
# ---------------------------------------------------------------------------

class _Params(ctypes.Structure):
    _fields_ = [
        ("num_steps", ctypes.c_uint32), ("method", ctypes.c_int32), ("cfg_mode", ctypes.c_int32),
        ("scale_text", ctypes.c_float), ("scale_caption", ctypes.c_float), ("scale_speaker", ctypes.c_float),
        ("min_t", ctypes.c_float), ("max_t", ctypes.c_float),
        ("has_truncation", ctypes.c_int32), ("truncation_factor", ctypes.c_float),
        ("has_temporal_rescale", ctypes.c_int32), ("rescale_k", ctypes.c_float), ("rescale_sigma", ctypes.c_float),
        ("has_speaker_kv", ctypes.c_int32), ("speaker_kv_scale", ctypes.c_float),
        ("speaker_kv_max_layers", ctypes.c_int32), ("has_speaker_kv_min_t", ctypes.c_int32),
        ("speaker_kv_min_t", ctypes.c_float), ("use_context_kv_cache", ctypes.c_int32),
    ]


class _Request(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int32), ("text_len", ctypes.c_int32),
        ("text_ids", ctypes.c_void_p), ("text_mask", ctypes.c_void_p),
        ("ref_len", ctypes.c_int32), ("ref_dim", ctypes.c_int32),
        ("ref_latent", ctypes.c_void_p), ("ref_mask", ctypes.c_void_p),
        ("caption_len", ctypes.c_int32), ("caption_ids", ctypes.c_void_p), ("caption_mask", ctypes.c_void_p),
        ("sequence_length", ctypes.c_int32), ("sequence_lengths", ctypes.c_void_p),
        ("initial_noise", ctypes.c_void_p), ("seed", ctypes.c_uint64), ("memory", ctypes.c_int32),
    ]


# Every symbol include/irodori_b200.h declares, with its signature.
_SIGNATURES = {
    "irt_last_error": (ctypes.c_char_p, []),
    "irt_version": (ctypes.c_char_p, []),
    "irt_sampler_params_default": (None, [ctypes.POINTER(_Params)]),
    "irt_sampler_params_validate": (ctypes.c_int, [ctypes.POINTER(_Params)]),
    "irt_engine_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "irt_engine_create_with_adapter": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int,
                                                      ctypes.POINTER(ctypes.c_void_p)]),
    "irt_engine_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "irt_engine_set_sampling": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(_Params)]),
    "irt_engine_set_default_sampling": (ctypes.c_int, [ctypes.c_void_p]),
    "irt_engine_get_sampling": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(_Params)]),
    "irt_engine_get_config": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,
                                             ctypes.POINTER(ctypes.c_size_t)]),
    "irt_engine_patched_latent_dim": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "irt_engine_use_speaker_condition": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "irt_engine_sample": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(_Request), ctypes.c_void_p, ctypes.c_int,
                                         ctypes.c_void_p]),
    "irt_engine_last_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                                             ctypes.POINTER(ctypes.c_int64)]),
    "irt_codec_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "irt_codec_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "irt_codec_sample_rate": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "irt_codec_hop_length": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "irt_codec_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "irt_codec_decode_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_void_p, ctypes.c_void_p]),
    "irt_codec_decode_ragged": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p, ctypes.c_int,
                                               ctypes.c_void_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load ``libirodori_b200.so`` (built by ``build.py``).  Raises if absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA library first (python irodori-tts-burn_b200/build.py)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != IRT_OK:
        msg = lib().irt_last_error().decode(errors="replace")
        raise _error_class(status)(status, msg)


def version() -> str:
    return lib().irt_version().decode()


# ---------------------------------------------------------------------------
# Sampler parameters (src/rf/params.rs:9-92)
# ---------------------------------------------------------------------------

@dataclass
class GuidanceConfig:
    """GuidanceConfig (src/rf/params.rs:9-35)."""
    mode: str = "independent"
    scale_text: float = 3.0
    scale_caption: float = 3.0
    scale_speaker: float = 5.0
    min_t: float = 0.5
    max_t: float = 1.0


@dataclass
class TemporalRescaleConfig:
    """TemporalRescaleConfig (src/rf/params.rs:40-46)."""
    k: float
    sigma: float


@dataclass
class SpeakerKvConfig:
    """SpeakerKvConfig (src/rf/params.rs:48-58)."""
    scale: float
    max_layers: Optional[int] = None
    min_t: Optional[float] = None


@dataclass
class SamplerParams:
    """SamplerParams (src/rf/params.rs:61-92)."""
    num_steps: int = 40
    method: str = "euler"
    guidance: GuidanceConfig = field(default_factory=GuidanceConfig)
    truncation_factor: Optional[float] = None
    temporal_rescale: Optional[TemporalRescaleConfig] = None
    speaker_kv: Optional[SpeakerKvConfig] = None
    use_context_kv_cache: bool = True

    def _to_c(self) -> _Params:
        p = _Params()
        lib().irt_sampler_params_default(ctypes.byref(p))
        if self.method not in METHODS:
            raise IrodoriError(4, f"Unsupported mode: unknown sampler method: {self.method!r}; "
                                  "expected euler, heun, or plms4")
        if self.guidance.mode not in MODES:
            raise IrodoriError(4, f"Unsupported mode: unknown cfg guidance mode: {self.guidance.mode!r}")
        p.num_steps = self.num_steps
        p.method = METHODS[self.method]
        g = self.guidance
        p.cfg_mode = MODES[g.mode]
        p.scale_text, p.scale_caption, p.scale_speaker = g.scale_text, g.scale_caption, g.scale_speaker
        p.min_t, p.max_t = g.min_t, g.max_t
        if self.truncation_factor is not None:
            p.has_truncation, p.truncation_factor = 1, self.truncation_factor
        if self.temporal_rescale is not None:
            p.has_temporal_rescale = 1
            p.rescale_k, p.rescale_sigma = self.temporal_rescale.k, self.temporal_rescale.sigma
        if self.speaker_kv is not None:
            s = self.speaker_kv
            p.has_speaker_kv, p.speaker_kv_scale = 1, s.scale
            p.speaker_kv_max_layers = -1 if s.max_layers is None else s.max_layers
            if s.min_t is not None:
                p.has_speaker_kv_min_t, p.speaker_kv_min_t = 1, s.min_t
        p.use_context_kv_cache = 1 if self.use_context_kv_cache else 0
        return p

    @classmethod
    def _from_c(cls, p: _Params) -> "SamplerParams":
        inv_m = {v: k for k, v in METHODS.items()}
        inv_g = {v: k for k, v in MODES.items()}
        return cls(
            num_steps=p.num_steps, method=inv_m[p.method],
            guidance=GuidanceConfig(inv_g[p.cfg_mode], p.scale_text, p.scale_caption, p.scale_speaker, p.min_t,
                                    p.max_t),
            truncation_factor=p.truncation_factor if p.has_truncation else None,
            temporal_rescale=TemporalRescaleConfig(p.rescale_k, p.rescale_sigma) if p.has_temporal_rescale else None,
            speaker_kv=SpeakerKvConfig(p.speaker_kv_scale,
                                       None if p.speaker_kv_max_layers < 0 else p.speaker_kv_max_layers,
                                       p.speaker_kv_min_t if p.has_speaker_kv_min_t else None)
            if p.has_speaker_kv else None,
            use_context_kv_cache=bool(p.use_context_kv_cache))

    def validate(self) -> None:
        """SamplerParams::validate (src/rf/params.rs:99-183)."""
        p = self._to_c()
        _check(lib().irt_sampler_params_validate(ctypes.byref(p)))


# ---------------------------------------------------------------------------
# Requests
# ---------------------------------------------------------------------------

@dataclass
class SamplingRequest:
    """SamplingRequest (src/rf/params.rs:234-247).  Arrays may be numpy arrays
    or torch tensors (all on the host, or all on the engine's GPU).
    ``sequence_lengths`` extends the reference for ragged batches."""
    text_ids: Any
    text_mask: Any
    sequence_length: int
    ref_latent: Any = None
    ref_mask: Any = None
    caption_ids: Any = None
    caption_mask: Any = None
    initial_noise: Any = None
    sequence_lengths: Optional[Sequence[int]] = None
    seed: int = 0


def _as_buffer(x, dtype: str, keep: list):
    """Return (pointer, shape, on_device) for a numpy array or torch tensor,
    converting dtype/contiguity as needed (the converted copy is kept alive in
    ``keep`` for the duration of the call)."""
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(x, torch.Tensor):
        tdt = {"int32": torch.int32, "uint8": torch.uint8, "float32": torch.float32}[dtype]
        if x.dtype == torch.bool:
            # one byte per element holding 0 / 1: the same buffer as uint8, no
            # conversion kernel on the device
            x = x.contiguous().view(torch.uint8)
        t = x.to(tdt).contiguous()
        keep.append(t)
        return t.data_ptr(), tuple(t.shape), t.is_cuda
    import numpy as np
    a = np.ascontiguousarray(np.asarray(x).astype(dtype, copy=False))
    keep.append(a)
    return a.ctypes.data, a.shape, False


def _stream_arg(stream, device: int, on_device: bool, owner):
    """Stream handle for one C call.

    An explicit ``stream`` (a torch stream or a raw ``cudaStream_t`` as an int)
    is used as is.  Without one, a call that reads or writes CUDA tensors runs
    on a side stream of ``owner`` (one per engine or codec) that first waits
    for torch's current stream on ``device``: work torch has queued on those
    tensors (their creation, a previous kernel) completes before the engine
    reads them.  The C calls return only after their own work is complete, so
    nothing has to be ordered on the way back.  Host-only calls pass NULL (the
    library's own stream)."""
    if stream is not None:
        return ctypes.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
    if not on_device:
        return None
    import torch
    side = getattr(owner, "_side_stream", None)
    if side is None:
        side = torch.cuda.Stream(device=device)
        owner._side_stream = side
    side.wait_stream(torch.cuda.current_stream(device))
    return ctypes.c_void_p(side.cuda_stream)


# ---------------------------------------------------------------------------
# Type-state builder (src/inference.rs:83-196)
# ---------------------------------------------------------------------------

class InferenceBuilder:
    """``InferenceBuilder<B, Unconfigured>``: created for a device; the only
    transition is ``load_weights``."""

    def __init__(self, device: int = 0):
        self._device = device

    def load_weights(self, path: str, precision: str = "bf16") -> "LoadedBuilder":
        """Load a safetensors checkpoint with ``config_json`` metadata
        (src/inference.rs:107-116).  ``precision`` = "bf16" (bf16 tensor cores)
        or "f32" (parity mode: f32 data, GEMMs on tf32 tensor cores over hi / lo
        operand halves with f32-level error)."""
        if precision not in PREC:
            raise IrodoriError(22, f"unknown precision {precision!r}")
        h = ctypes.c_void_p()
        _check(lib().irt_engine_create(self._device, str(path).encode(), PREC[precision], ctypes.byref(h)))
        return LoadedBuilder(_Handle(h), self._device, precision)

    def load_weights_with_adapter(self, path: str, adapter_dir: str, precision: str = "bf16") -> "LoadedBuilder":
        """Load a checkpoint and merge a PEFT LoRA adapter directory
        (adapter_config.json + adapter_model.safetensors) into its weights at
        load (src/inference.rs:118-139)."""
        if precision not in PREC:
            raise IrodoriError(22, f"unknown precision {precision!r}")
        h = ctypes.c_void_p()
        _check(lib().irt_engine_create_with_adapter(self._device, str(path).encode(), str(adapter_dir).encode(),
                                                    PREC[precision], ctypes.byref(h)))
        return LoadedBuilder(_Handle(h), self._device, precision)


class _Handle:
    def __init__(self, h: ctypes.c_void_p):
        self.h = h

    def __del__(self):
        if self.h and _lib is not None:
            _lib.irt_engine_destroy(self.h)
            self.h = None


class LoadedBuilder:
    """``InferenceBuilder<B, Loaded>`` (src/inference.rs:143-165)."""

    def __init__(self, handle: _Handle, device: int, precision: str):
        self._h, self._device, self._precision = handle, device, precision

    def model_config(self) -> dict:
        return _engine_config(self._h)

    def with_sampling(self, params: SamplerParams) -> "ReadyBuilder":
        p = params._to_c()
        _check(lib().irt_engine_set_sampling(self._h.h, ctypes.byref(p)))
        return ReadyBuilder(self._h, self._device, self._precision)

    def with_default_sampling(self) -> "ReadyBuilder":
        return self.with_sampling(SamplerParams())


class ReadyBuilder:
    """``InferenceBuilder<B, Ready>`` (src/inference.rs:167-196)."""

    def __init__(self, handle: _Handle, device: int, precision: str):
        self._h, self._device, self._precision = handle, device, precision

    def with_sampling(self, params: SamplerParams) -> "ReadyBuilder":
        p = params._to_c()
        _check(lib().irt_engine_set_sampling(self._h.h, ctypes.byref(p)))
        return self

    def build(self) -> "InferenceEngine":
        return InferenceEngine(self._h, self._device, self._precision)


def _engine_config(h: _Handle) -> dict:
    n = ctypes.c_size_t()
    _check(lib().irt_engine_get_config(h.h, None, 0, ctypes.byref(n)))
    buf = ctypes.create_string_buffer(n.value)
    _check(lib().irt_engine_get_config(h.h, buf, n.value, ctypes.byref(n)))
    return json.loads(buf.value.decode())


class InferenceEngine:
    """``InferenceEngine<B>`` (src/inference.rs:203-254)."""

    def __init__(self, handle: _Handle, device: int, precision: str):
        self._h, self._device, self._precision = handle, device, precision

    # accessors (src/inference.rs:229-253, src/model/optimized.rs:133-141)
    def model_config(self) -> dict:
        return _engine_config(self._h)

    def sampling_params(self) -> SamplerParams:
        p = _Params()
        _check(lib().irt_engine_get_sampling(self._h.h, ctypes.byref(p)))
        return SamplerParams._from_c(p)

    def device(self) -> int:
        return self._device

    def precision(self) -> str:
        return self._precision

    def patched_latent_dim(self) -> int:
        v = ctypes.c_int32()
        _check(lib().irt_engine_patched_latent_dim(self._h.h, ctypes.byref(v)))
        return v.value

    def use_speaker_condition(self) -> bool:
        v = ctypes.c_int32()
        _check(lib().irt_engine_use_speaker_condition(self._h.h, ctypes.byref(v)))
        return bool(v.value)

    def with_sampling(self, params: SamplerParams) -> "InferenceEngine":
        p = params._to_c()
        _check(lib().irt_engine_set_sampling(self._h.h, ctypes.byref(p)))
        return self

    def last_stats(self):
        """(DiT row-forwards, kernel launches) of the last ``sample`` call."""
        a, b = ctypes.c_int64(), ctypes.c_int64()
        _check(lib().irt_engine_last_stats(self._h.h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def sample(self, request: SamplingRequest, out=None, stream=None):
        """Run the RF sampler (src/inference.rs:222-227).  Returns the latent
        ``[batch, sequence_length, patched_latent_dim]`` as a numpy array, or
        writes into ``out`` (a torch tensor, host or device) and returns it."""
        keep: list = []
        r = _Request()
        ids_p, ids_shape, dev0 = _as_buffer(request.text_ids, "int32", keep)
        if len(ids_shape) != 2:
            raise IrodoriError(2, "Shape mismatch: text_ids must be [batch, text_len]")
        B, T = ids_shape
        m_p, m_shape, dev1 = _as_buffer(request.text_mask, "uint8", keep)
        if tuple(m_shape) != (B, T):
            raise IrodoriError(2, "Shape mismatch: text_mask must match text_ids")
        devs = [dev0, dev1]
        r.batch, r.text_len, r.text_ids, r.text_mask = B, T, ids_p, m_p
        if request.ref_latent is not None and request.ref_mask is not None:
            rl_p, rl_shape, d2 = _as_buffer(request.ref_latent, "float32", keep)
            rm_p, rm_shape, d3 = _as_buffer(request.ref_mask, "uint8", keep)
            if len(rl_shape) != 3 or rl_shape[0] != B or tuple(rm_shape) != tuple(rl_shape[:2]):
                raise IrodoriError(2, "Shape mismatch: ref_latent [B,T,D] / ref_mask [B,T]")
            r.ref_len, r.ref_dim, r.ref_latent, r.ref_mask = rl_shape[1], rl_shape[2], rl_p, rm_p
            devs += [d2, d3]
        if request.caption_ids is not None and request.caption_mask is not None:
            c_p, c_shape, d4 = _as_buffer(request.caption_ids, "int32", keep)
            cm_p, cm_shape, d5 = _as_buffer(request.caption_mask, "uint8", keep)
            if len(c_shape) != 2 or c_shape[0] != B or tuple(cm_shape) != tuple(c_shape):
                raise IrodoriError(2, "Shape mismatch: caption_ids / caption_mask")
            r.caption_len, r.caption_ids, r.caption_mask = c_shape[1], c_p, cm_p
            devs += [d4, d5]
        P = self.patched_latent_dim()
        S = int(request.sequence_length)
        r.sequence_length = S
        if request.sequence_lengths is not None:
            import numpy as np
            sl = np.ascontiguousarray(np.asarray(request.sequence_lengths, dtype=np.int32))
            if sl.shape != (B,):
                raise IrodoriError(2, "Shape mismatch: sequence_lengths must be [batch]")
            keep.append(sl)
            r.sequence_lengths = sl.ctypes.data
        if request.initial_noise is not None:
            n_p, n_shape, d6 = _as_buffer(request.initial_noise, "float32", keep)
            if tuple(n_shape) != (B, S, P):
                raise IrodoriError(2, f"Shape mismatch: initial_noise must be [{B}, {S}, {P}], got {list(n_shape)}")
            r.initial_noise = n_p
            devs.append(d6)
        if any(devs) and not all(devs):
            raise IrodoriError(22, "request arrays must be all on the host or all on the GPU")
        r.memory = MEM_DEVICE if all(devs) else MEM_HOST
        r.seed = int(request.seed)
        import numpy as np
        if out is None:
            out = np.empty((B, S, P), dtype=np.float32)
        if isinstance(out, np.ndarray):
            if out.shape != (B, S, P) or out.dtype != np.float32 or not out.flags["C_CONTIGUOUS"]:
                raise IrodoriError(2, "Shape mismatch: out must be a contiguous float32 [B, S, P] array")
            res = out
            o_p, o_mem = out.ctypes.data, MEM_HOST
        else:
            if tuple(out.shape) != (B, S, P) or not out.is_contiguous():
                raise IrodoriError(2, "Shape mismatch: out must be a contiguous [B, S, P] tensor")
            res = out
            o_p, o_mem = out.data_ptr(), MEM_DEVICE if out.is_cuda else MEM_HOST
        st = _stream_arg(stream, self._device, r.memory == MEM_DEVICE or o_mem == MEM_DEVICE, self)
        _check(lib().irt_engine_sample(self._h.h, ctypes.byref(r), ctypes.c_void_p(o_p), o_mem, st))
        return res


# ---------------------------------------------------------------------------
# DACVAE codec (src/codec/weights.rs:27-33, src/codec/model.rs:18-65)
# ---------------------------------------------------------------------------

class DacVaeCodec:
    """Decoder side of ``DacVaeCodec<B>``."""

    def __init__(self, handle: ctypes.c_void_p, device: int):
        self._h, self._device = handle, device

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.irt_codec_destroy(self._h)
            self._h = None

    def sample_rate(self) -> int:
        v = ctypes.c_int32()
        _check(lib().irt_codec_sample_rate(self._h, ctypes.byref(v)))
        return v.value

    def hop_length(self) -> int:
        v = ctypes.c_int32()
        _check(lib().irt_codec_hop_length(self._h, ctypes.byref(v)))
        return v.value

    def decode(self, latent, out=None, stream=None, lengths=None):
        """``[B, T, 32]`` latent -> ``[B, 1, T * hop_length]`` waveform.

        ``lengths`` (extension, ``irt_codec_decode_ragged``): valid latent
        frames per utterance; each utterance is decoded as if alone at its
        length and samples past ``lengths[b] * hop_length`` are zero."""
        keep: list = []
        p, shape, dev = _as_buffer(latent, "float32", keep)
        if len(shape) != 3 or shape[2] != 32:
            raise IrodoriError(2, "Shape mismatch: latent must be [B, T, 32]")
        B, T, _ = shape
        n = T * self.hop_length()
        if out is None:
            import numpy as np
            res = np.empty((B, 1, n), dtype=np.float32)
            o_p, o_mem = res.ctypes.data, MEM_HOST
            if dev:
                raise IrodoriError(22, "device latent needs a device `out` tensor")
        else:
            res = out
            o_p, o_mem = out.data_ptr(), MEM_DEVICE if out.is_cuda else MEM_HOST
            if o_mem != (MEM_DEVICE if dev else MEM_HOST):
                raise IrodoriError(22, "latent and out must live in the same memory")
        st = _stream_arg(stream, self._device, bool(dev) or o_mem == MEM_DEVICE, self)
        if lengths is None:
            _check(lib().irt_codec_decode(self._h, ctypes.c_void_p(p), B, T, ctypes.c_void_p(o_p),
                                          MEM_DEVICE if dev else MEM_HOST, st))
        else:
            lens = [int(v) for v in lengths]
            if len(lens) != B:
                raise IrodoriError(2, f"Shape mismatch: {len(lens)} lengths for a batch of {B}")
            arr = (ctypes.c_int32 * B)(*lens)
            _check(lib().irt_codec_decode_ragged(self._h, ctypes.c_void_p(p), B, T, arr, ctypes.c_void_p(o_p),
                                                 MEM_DEVICE if dev else MEM_HOST, st))
        return res


def decode_noalloc(codec: DacVaeCodec, latent, wav, stream=None):
    """Allocation-free decode (``irt_codec_decode_noalloc``) for callers that
    cannot allocate device memory mid-decode (streaming loops that cannot
    absorb cudaMalloc/cudaFree synchronisation, hosts whose allocator owns the
    free HBM).  ``latent`` [B, T, 32] and ``wav`` [B, 1, T * hop] are
    contiguous float32 CUDA tensors on the codec's GPU; nothing is converted or
    copied here (a conversion would allocate).  B * T is limited by a fixed
    16 MiB device scratch array (7 frames for the full-width DACVAE).  Calls
    that overlap on the GPU race on that array.  With ``stream=None`` the call
    is ordered after torch's current stream.  Returns ``wav``."""
    import torch
    for name, t in (("latent", latent), ("wav", wav)):
        if not isinstance(t, torch.Tensor):
            raise IrodoriError(22, f"decode_noalloc: {name} must be a torch tensor")
        if t.dtype != torch.float32:
            raise IrodoriError(9, f"decode_noalloc: {name} must be float32, got {t.dtype}")
        if not t.is_contiguous():
            raise IrodoriError(22, f"decode_noalloc: {name} must be contiguous")
    if latent.dim() != 3 or latent.shape[2] != 32:
        raise IrodoriError(2, "Shape mismatch: latent must be [B, T, 32]")
    B, T, _ = latent.shape
    if tuple(wav.shape) != (B, 1, T * codec.hop_length()):
        raise IrodoriError(2, "Shape mismatch: latent [B, T, 32] and wav [B, 1, T * hop]")
    for name, t in (("latent", latent), ("wav", wav)):
        if not t.is_cuda or t.device.index != codec._device:
            raise IrodoriError(22, f"decode_noalloc: {name} must be a CUDA tensor on the codec's GPU "
                                   f"(cuda:{codec._device}), got {t.device}")
    st = _stream_arg(stream, codec._device, True, codec)
    _check(lib().irt_codec_decode_noalloc(codec._h, ctypes.c_void_p(latent.data_ptr()), B, T,
                                          ctypes.c_void_p(wav.data_ptr()), st))
    return wav


def load_codec(path: str, device: int = 0, precision: str = "f32") -> DacVaeCodec:
    """load_codec (src/codec/weights.rs:27-33).  ``precision`` = "f32" (f32 data,
    convolutions on tf32 tensor cores over hi / lo operand halves) or "bf16"
    (bf16 tensor-core convolutions)."""
    h = ctypes.c_void_p()
    _check(lib().irt_codec_create(device, str(path).encode(), PREC[precision], ctypes.byref(h)))
    return DacVaeCodec(h, device)


__all__ = [
    "InferenceBuilder", "LoadedBuilder", "ReadyBuilder", "InferenceEngine", "SamplerParams", "GuidanceConfig",
    "TemporalRescaleConfig", "SpeakerKvConfig", "SamplingRequest", "DacVaeCodec", "load_codec", "IrodoriError",
    "ConfigError", "StateError", "lib", "version", "LIB_PATH",
]
