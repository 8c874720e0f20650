"""Python mirror of the reference backend interface over the C ABI.

``CudaEngine`` offers the methods of ``minigo::InferenceEngine``
(include/inference_engine.h:14-41) - ``load_model``, ``predict``,
``predict_batch``, ``backend_name`` and the ``board_size`` /
``input_channels`` / ``num_filters`` / ``num_res_blocks`` metadata - with the
same argument meaning and error behaviour (failures raise ``RuntimeError``
where the C++ engines throw ``std::runtime_error``).  Every call goes through
libminigo_cuda.so (include/minigo_cuda.h); there is no CPU fallback: if the
library is missing or no sm_100 GPU is present, construction fails.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build

PREC = {"bf16": 0, "fp16": 1, "fp32": 2}
FLAG_EIGEN_COMPAT = 1

_LIB = None


class mg_tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dims", ctypes.POINTER(ctypes.c_int64)),
                ("ndims", ctypes.c_int), ("data", ctypes.c_void_p)]


def lib() -> ctypes.CDLL:
    """Loads libminigo_cuda.so; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        path = build.CUDA_LIB
        if not os.path.exists(path):
            raise RuntimeError(f"CUDA extension {path} is missing: run `python -m alphazero_b200.build`")
        L = ctypes.CDLL(path)
        vp, ci, fp = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
        L.mg_create.argtypes = [ci, ci]
        L.mg_create.restype = vp
        L.mg_create_error.restype = ctypes.c_char_p
        L.mg_destroy.argtypes = [vp]
        L.mg_last_error.argtypes = [vp]
        L.mg_last_error.restype = ctypes.c_char_p
        L.mg_load_onnx.argtypes = [vp, ctypes.c_char_p]
        L.mg_load_weights.argtypes = [vp, ctypes.POINTER(mg_tensor), ci]
        L.mg_get_info.argtypes = [vp] + [ctypes.POINTER(ci)] * 5
        L.mg_set_precision.argtypes = [vp, ci]
        L.mg_set_max_batch.argtypes = [vp, ci]
        L.mg_forward.argtypes = [vp, fp, ci, fp, fp, fp]
        L.mg_forward_device.argtypes = [vp, fp, ci, fp, fp, fp]
        L.mg_forward_device_noalloc.argtypes = [vp, fp, ci, fp, fp, fp]
        L.mg_forward_packed.argtypes = [vp, fp, ci, fp, fp, fp]
        L.mg_forward_history.argtypes = [vp, fp, ci, fp, fp, fp]
        L.mg_history_words.argtypes = [vp]
        L.mg_submit_packed.argtypes = [vp, fp, ci, fp, fp, ctypes.POINTER(ci)]
        L.mg_wait_submitted.argtypes = [vp, ci]
        L.mg_words_per_position.argtypes = [vp]
        L.mg_pack_states.argtypes = [fp, ci, ci, fp]
        L.mg_synchronize.argtypes = [vp]
        L.mg_stream.argtypes = [vp]
        L.mg_stream.restype = vp
        L.mg_launch_conv.argtypes = [vp, ci, ci, ci]
        L.mg_launch_trunk.argtypes = [vp, ci, ci]
        L.mg_launches_per_forward.argtypes = [vp, ci]
        for f in ("mg_load_onnx", "mg_load_weights", "mg_get_info", "mg_set_precision",
                  "mg_set_max_batch", "mg_forward", "mg_forward_device", "mg_forward_device_noalloc",
                  "mg_forward_packed", "mg_forward_history", "mg_history_words",
                  "mg_submit_packed", "mg_wait_submitted",
                  "mg_words_per_position", "mg_pack_states", "mg_synchronize",
                  "mg_launch_conv", "mg_launch_trunk", "mg_launches_per_forward"):
            getattr(L, f).restype = ci
        _LIB = L
    return _LIB


def pack_states(states) -> np.ndarray:
    """[n, size] binary fp32 planes -> [n, ceil(size / 32)] uint32 words of
    the packed wire format (bit j % 32 of word j / 32), via mg_pack_states."""
    x = np.ascontiguousarray(states, dtype=np.float32)
    n, size = x.shape
    out = np.empty((n, (size + 31) // 32), np.uint32)
    if lib().mg_pack_states(x.ctypes.data, n, size, out.ctypes.data) != 0:
        raise ValueError("states are not binary planes (values other than 0 and 1)")
    return out


class CudaEngine:
    """One network resident on one GPU (not thread-safe, like the reference
    engines: one evaluator thread drives one engine)."""

    def __init__(self, device: int = 0, precision: str = "bf16", eigen_compat: bool = False,
                 max_batch: int = 1024):
        L = lib()
        self._L = L
        h = L.mg_create(device, FLAG_EIGEN_COMPAT if eigen_compat else 0)
        if not h:
            raise RuntimeError("mg_create failed: " + L.mg_create_error().decode())
        self._h = ctypes.c_void_p(h)
        self.device = device
        self.board_size = 9
        self.input_channels = 17
        self.num_filters = 64
        self.num_res_blocks = 5
        self.action_size = 82
        self._check(L.mg_set_max_batch(self._h, max_batch))
        self.set_precision(precision)

    # -- plumbing --
    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(self._L.mg_last_error(self._h).decode() or f"error {rc}")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.mg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _refresh_info(self) -> None:
        v = [ctypes.c_int() for _ in range(5)]
        self._check(self._L.mg_get_info(self._h, *[ctypes.byref(x) for x in v]))
        (self.board_size, self.input_channels, self.num_filters, self.num_res_blocks,
         self.action_size) = (x.value for x in v)

    # -- InferenceEngine interface --
    def load_model(self, model_path: str) -> None:
        self._check(self._L.mg_load_onnx(self._h, os.fsencode(model_path)))
        self._refresh_info()

    def load_state_dict(self, sd) -> None:
        """Loads named fp32 arrays directly (non-fp32 entries are skipped)."""
        keep = [(k, np.ascontiguousarray(v, dtype=np.float32)) for k, v in sd.items()
                if np.asarray(v).dtype == np.float32]
        arr = (mg_tensor * len(keep))()
        hold = []
        for i, (k, v) in enumerate(keep):
            dims = (ctypes.c_int64 * max(1, v.ndim))(*v.shape)
            hold.append((dims, v))
            arr[i].name = k.encode()
            arr[i].dims = dims
            arr[i].ndims = v.ndim
            arr[i].data = v.ctypes.data
        self._check(self._L.mg_load_weights(self._h, arr, len(keep)))
        self._refresh_info()

    def backend_name(self) -> str:
        return "cuda"

    def set_precision(self, precision: str) -> None:
        self._check(self._L.mg_set_precision(self._h, PREC[precision]))
        self.precision = precision

    def forward(self, states, want_logits: bool = True):
        """states [n, 17*B*B] float32 (host) -> (probs [n, A], values [n],
        logits [n, A] or None)."""
        x = np.ascontiguousarray(states, dtype=np.float32)
        n = x.shape[0] if x.ndim > 1 else (1 if x.size else 0)
        A = self.action_size
        probs = np.empty((n, A), np.float32)
        vals = np.empty((n,), np.float32)
        logits = np.empty((n, A), np.float32) if want_logits else None
        if n:
            self._check(self._L.mg_forward(self._h, x.ctypes.data, n, probs.ctypes.data,
                                           vals.ctypes.data,
                                           logits.ctypes.data if want_logits else None))
        return probs, vals, logits

    def forward_packed(self, bits, n: int, want_logits: bool = False, out=None):
        """Bit-packed wire format (see pack_states): bits holds n x
        words_per_position() uint32 words.  `out` may supply (probs, values)
        arrays to fill (e.g. pinned); returns (probs, values, logits)."""
        b = np.ascontiguousarray(bits, dtype=np.uint32)
        A = self.action_size
        probs, vals = out if out is not None else (np.empty((n, A), np.float32),
                                                    np.empty((n,), np.float32))
        logits = np.empty((n, A), np.float32) if want_logits else None
        if n:
            self._check(self._L.mg_forward_packed(self._h, b.ctypes.data, n, probs.ctypes.data,
                                                  vals.ctypes.data,
                                                  logits.ctypes.data if want_logits else None))
        return probs, vals, logits

    def words_per_position(self) -> int:
        return self._L.mg_words_per_position(self._h)

    def forward_history(self, hist, n: int, want_logits: bool = False, out=None):
        """History wire format (include/minigo_cuda.h, mg_forward_history):
        hist holds n x history_words() uint32 words, the last 8 boards of
        each position at 2 bits per point; the planes are expanded on the
        device.  Returns (probs, values, logits) like forward_packed."""
        h = np.ascontiguousarray(hist, dtype=np.uint32)
        A = self.action_size
        probs, vals = out if out is not None else (np.empty((n, A), np.float32),
                                                    np.empty((n,), np.float32))
        logits = np.empty((n, A), np.float32) if want_logits else None
        if n:
            self._check(self._L.mg_forward_history(self._h, h.ctypes.data, n, probs.ctypes.data,
                                                   vals.ctypes.data,
                                                   logits.ctypes.data if want_logits else None))
        return probs, vals, logits

    def submit_packed(self, bits, n: int, probs, values) -> int:
        """mg_submit_packed: enqueues n bit-packed positions from page-locked
        `bits` with results into the page-locked arrays probs [n, A] and
        values [n]; returns a ticket for wait_submitted.  The arrays must
        stay alive (and unread) until then."""
        t = ctypes.c_int(-1)
        self._check(self._L.mg_submit_packed(self._h, bits.ctypes.data, n, probs.ctypes.data,
                                             values.ctypes.data, ctypes.byref(t)))
        return t.value

    def wait_submitted(self, ticket: int) -> None:
        rc = self._L.mg_wait_submitted(self._h, ticket)
        if rc != 0:
            raise RuntimeError(f"mg_wait_submitted failed ({rc})")

    def history_words(self) -> int:
        return self._L.mg_history_words(self._h)

    def predict(self, state):
        """(softmaxed policy, value in [-1, 1]) for one flat state."""
        p, v, _ = self.forward(np.asarray(state, np.float32).reshape(1, -1), want_logits=False)
        return p[0], float(v[0])

    def predict_batch(self, states):
        """List of (policy, value); an empty batch returns []."""
        if len(states) == 0:
            return []
        p, v, _ = self.forward(np.stack([np.asarray(s, np.float32) for s in states]),
                               want_logits=False)
        return [(p[i], float(v[i])) for i in range(len(states))]

    # -- device-resident path and measurement hooks --
    def forward_device(self, d_states: int, n: int, d_policy: int, d_value: int,
                       d_logits: int | None = None) -> None:
        self._check(self._L.mg_forward_device(self._h, d_states, n, d_policy, d_value, d_logits))

    def forward_device_noalloc(self, d_states: int, n: int, d_policy: int, d_value: int,
                               d_logits: int | None = None) -> None:
        """As forward_device, with every intermediate buffer taken from the
        library's fixed per-device scratch arena (no device allocation);
        blocks until the outputs are written."""
        self._check(self._L.mg_forward_device_noalloc(self._h, d_states, n, d_policy, d_value,
                                                      d_logits))

    def synchronize(self) -> None:
        self._check(self._L.mg_synchronize(self._h))

    def stream_handle(self) -> int:
        return self._L.mg_stream(self._h)

    def launch_conv(self, n: int, layer: int, reps: int) -> None:
        self._check(self._L.mg_launch_conv(self._h, n, layer, reps))

    def launch_trunk(self, n: int, reps: int) -> None:
        self._check(self._L.mg_launch_trunk(self._h, n, reps))

    def launches_per_forward(self, n: int) -> int:
        return self._L.mg_launches_per_forward(self._h, n)
