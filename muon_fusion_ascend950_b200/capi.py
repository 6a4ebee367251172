"""ctypes binding of the C ABI in include/muon_polar_sm100.h.

This is the binding a ctypes-based caller of the reference's launchers would
add (csrc/muon_polar_step_binding.cpp:65-70 declares those).  The tests use
it to drive the kernels through the exact boundary other languages see, and
the multi-GPU drivers use the per-stage entry points.  Loading the library
needs no GPU; every compute call needs an sm_100 device.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

LIB_FILENAME = "libmuon_polar_sm100.so"

# Every entry point declared in include/muon_polar_sm100.h:
# name -> (restype, argtypes)
_I64 = ctypes.c_int64
_VP = ctypes.c_void_p
SIGNATURES = {
    "muon_polar_abi_version": (ctypes.c_int, []),
    "muon_polar_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "muon_polar_padded_rows": (_I64, [_I64]),
    "muon_polar_workspace_bytes": (ctypes.c_size_t, [_I64, _I64]),
    "muon_polar_scratch_bytes": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "muon_polar_scratch_init": (ctypes.c_int, [_VP, ctypes.c_size_t, _VP]),
    "muon_polar_gram_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64, _VP,
                                             ctypes.c_size_t, _VP]),
    "muon_polar_gram_static_scratch_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64,
                                                            _VP]),
    "muon_polar_gram_f32_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64, _VP,
                                                 ctypes.c_size_t, _VP]),
    "muon_polar_gram_f32_band_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64, _I64,
                                                      _I64, ctypes.c_int, _VP, ctypes.c_size_t,
                                                      _VP]),
    "muon_polar_poly_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, ctypes.c_float,
                                             ctypes.c_float, _VP, ctypes.c_size_t, _VP]),
    "muon_polar_poly_rows_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64,
                                                  ctypes.c_float, ctypes.c_float, _VP]),
    "muon_polar_apply_sm100": (ctypes.c_int, [_VP, _VP, _VP, _I64, _I64, _I64, _I64,
                                              _I64, ctypes.c_float, _VP]),
    "muon_polar_step_sm100": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_size_t, _VP,
                                             ctypes.c_size_t, _I64, _I64, _I64, _I64, _I64,
                                             ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                             _VP]),
    "muon_polar_gram_t_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64, _VP,
                                               ctypes.c_size_t, _VP]),
    "muon_polar_apply_t_sm100": (ctypes.c_int, [_VP, _VP, _VP, _I64, _I64, _I64, _I64,
                                                _I64, ctypes.c_float, _VP]),
    "muon_polar_step_t_sm100": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_size_t, _VP,
                                               ctypes.c_size_t, _I64, _I64, _I64, _I64, _I64,
                                               ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                               _VP]),
    "muon_polar_steps_sm100": (ctypes.c_int, [_VP, _VP, _VP, _VP, _I64, _VP, ctypes.c_size_t,
                                              _VP, ctypes.c_size_t, _I64, _I64, _I64, _I64,
                                              _I64, ctypes.POINTER(ctypes.c_float),
                                              ctypes.c_int, _VP]),
    "muon_polar_express_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "muon_polar_express_sm100": (ctypes.c_int, [_VP, ctypes.c_int, _I64, _VP, _I64, _VP,
                                                ctypes.c_size_t, _VP, ctypes.c_size_t, _I64,
                                                _I64, _I64, ctypes.POINTER(ctypes.c_float),
                                                ctypes.c_int, ctypes.c_int, _VP]),
    "muon_polar_update_sm100": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, _VP, ctypes.c_size_t,
                                         _VP, ctypes.c_size_t, _I64, _I64, _I64,
                                         ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_float,
                                         ctypes.POINTER(ctypes.c_float), ctypes.c_int, _VP]),
    "muon_polar_update_launch_count": (ctypes.c_uint64, []),
    "muon_polar_cast_f32_bf16_sm100": (ctypes.c_int, [_VP, _VP, _I64, _VP]),
    "muon_polar_read_device_status": (ctypes.c_int, [ctypes.c_int,
                                                     ctypes.POINTER(ctypes.c_uint32),
                                                     ctypes.c_int]),
    "muon_polar_set_kernel_policy": (ctypes.c_int, [ctypes.c_int]),
    "muon_polar_set_step_mode": (ctypes.c_int, [ctypes.c_int]),
    "muon_polar_set_split_mode": (ctypes.c_int, [ctypes.c_int]),
    "muon_polar_set_halves_mode": (ctypes.c_int, [ctypes.c_int]),
    "muon_polar_set_stage_mode": (ctypes.c_int, [ctypes.c_int]),
    "muon_polar_device_pairs": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "muon_polar_launch_count": (ctypes.c_uint64, []),
    "muon_polar_tensor_map_encodes": (ctypes.c_uint64, []),
    "muon_polar_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64,
                                                    ctypes.POINTER(ctypes.c_uint64)]),
    "muon_polar_set_static_scratch_limit": (ctypes.c_size_t, [ctypes.c_size_t]),
    "muon_polar_decode_tile": (ctypes.c_int, [_I64, ctypes.c_int, _I64, _I64, _I64, _I64,
                                              ctypes.POINTER(_I64)]),
    "muon_polar_check_address_cache": (ctypes.c_int, []),
    "muon_polar_packed_units": (_I64, [_I64]),
    "muon_polar_gram_f32_packed_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64, _VP,
                                                        ctypes.c_size_t, _VP]),
    "muon_polar_poly_packed_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I64,
                                                    ctypes.c_float, ctypes.c_float, _VP]),
    "muon_polar_unpack_sym_sm100": (ctypes.c_int, [_VP, _VP, _I64, _I64, _VP]),
}

WATCHDOG_PRODUCER = 0x1
WATCHDOG_MMA = 0x2
WATCHDOG_EPILOGUE = 0x4
WATCHDOG_DRAIN = 0x8
WATCHDOG_DEPENDENCY = 0x10


class MuonPolarError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, func: str, status: int, text: str):
        super().__init__(f"{func} failed, status={status}: {text}")
        self.status = status


def library_path() -> Path:
    configured = os.environ.get("MUON_POLAR_SM100_LIBRARY")
    if configured:
        return Path(configured).expanduser().resolve()
    return Path(__file__).resolve().parent / LIB_FILENAME


def _nbytes(t) -> int:
    return t.numel() * t.element_size()


def _scratch(scratch):
    if scratch is None or scratch.numel() == 0:
        return None, 0
    return scratch.data_ptr(), _nbytes(scratch)


class CAPI:
    """Typed access to libmuon_polar_sm100.so."""

    def __init__(self, path: Optional[Path] = None):
        path = Path(path) if path is not None else library_path()
        if not path.is_file():
            raise RuntimeError(
                f"{path} is missing; build it with `python -m muon_fusion_ascend950_b200.build`")
        self.path = path
        self.lib = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = restype
            fn.argtypes = argtypes

    # -------------------------------------------------------------- helpers
    def status_string(self, status: int) -> str:
        return self.lib.muon_polar_status_string(int(status)).decode()

    def _check(self, func: str, status: int) -> None:
        if status != 0:
            raise MuonPolarError(func, status, self.status_string(status))

    @staticmethod
    def _stream(stream) -> int:
        import torch

        if stream is None:
            stream = torch.cuda.current_stream()
        return int(getattr(stream, "cuda_stream", stream))

    def abi_version(self) -> int:
        return int(self.lib.muon_polar_abi_version())

    def padded_rows(self, m: int) -> int:
        return int(self.lib.muon_polar_padded_rows(int(m)))

    def workspace_bytes(self, batch: int, m: int) -> int:
        return int(self.lib.muon_polar_workspace_bytes(int(batch), int(m)))

    def set_kernel_policy(self, policy: int) -> int:
        """0 = by size, 1 = always CTA pairs, 2 = always single-CTA; returns
        the previous policy."""
        prev = int(self.lib.muon_polar_set_kernel_policy(int(policy)))
        if prev < 0:
            raise MuonPolarError("muon_polar_set_kernel_policy", prev, self.status_string(prev))
        return prev

    def set_step_mode(self, mode: int) -> int:
        """0 = by size, 1 = always one fused launch, 2 = always three kernels;
        returns the previous mode."""
        prev = int(self.lib.muon_polar_set_step_mode(int(mode)))
        if prev < 0:
            raise MuonPolarError("muon_polar_set_step_mode", prev, self.status_string(prev))
        return prev

    def set_split_mode(self, mode: int) -> int:
        """0 = by size, 1 = whenever the device has room, 2 = never; returns
        the previous mode."""
        prev = int(self.lib.muon_polar_set_split_mode(int(mode)))
        if prev < 0:
            raise MuonPolarError("muon_polar_set_split_mode", prev, self.status_string(prev))
        return prev

    def set_halves_mode(self, mode: int) -> int:
        """0 = by size (whenever the column halves fit in one round), 1 = the
        same, 2 = never; returns the previous mode."""
        prev = int(self.lib.muon_polar_set_halves_mode(int(mode)))
        if prev < 0:
            raise MuonPolarError("muon_polar_set_halves_mode", prev, self.status_string(prev))
        return prev

    def set_stage_mode(self, mode: int) -> int:
        """0 = by size (K = 192 stages for the single-CTA bf16 Gram when
        they cover at most 4% more K), 1 = whenever no split-K is planned,
        2 = never; returns the previous mode."""
        prev = int(self.lib.muon_polar_set_stage_mode(int(mode)))
        if prev < 0:
            raise MuonPolarError("muon_polar_set_stage_mode", prev, self.status_string(prev))
        return prev

    def device_pairs(self) -> int:
        pairs = ctypes.c_int(0)
        self._check("muon_polar_device_pairs", self.lib.muon_polar_device_pairs(ctypes.byref(pairs)))
        return int(pairs.value)

    def launch_count(self) -> int:
        return int(self.lib.muon_polar_launch_count())

    def tensor_map_encodes(self) -> int:
        return int(self.lib.muon_polar_tensor_map_encodes())

    def read_device_status(self, device: int, clear: bool = True) -> int:
        flags = ctypes.c_uint32(0)
        self._check("muon_polar_read_device_status",
                    self.lib.muon_polar_read_device_status(int(device), ctypes.byref(flags),
                                                           1 if clear else 0))
        return int(flags.value)

    def set_wait_limit_ns(self, limit_ns: int) -> int:
        """Limit of the kernels' bounded waits on the current device; returns
        the previous limit."""
        prev = ctypes.c_uint64(0)
        self._check("muon_polar_set_wait_limit_ns",
                    self.lib.muon_polar_set_wait_limit_ns(int(limit_ns), ctypes.byref(prev)))
        return int(prev.value)

    def set_static_scratch_limit(self, nbytes: int) -> int:
        """Budget of gram_static_scratch in bytes of the built-in array (0:
        all of it); returns the previous budget."""
        return int(self.lib.muon_polar_set_static_scratch_limit(int(nbytes)))

    def decode_tile(self, tile: int, symmetric: bool, tiles_m: int, tiles_n: int,
                    tiles_per_batch: int, first_row: int = 0):
        """(batch, tile row, tile col) of linear tile index `tile` in the
        kernels' work-item order (host copy of the device enumeration)."""
        out = (_I64 * 3)()
        self._check("muon_polar_decode_tile", self.lib.muon_polar_decode_tile(
            int(tile), 1 if symmetric else 0, int(tiles_m), int(tiles_n), int(tiles_per_batch),
            int(first_row), out))
        return int(out[0]), int(out[1]), int(out[2])

    def check_address_cache(self) -> int:
        return int(self.lib.muon_polar_check_address_cache())

    def scratch_bytes(self, batch: int, m: int, n: int) -> int:
        return int(self.lib.muon_polar_scratch_bytes(int(batch), int(m), int(n)))

    def scratch_init(self, scratch, stream=None) -> None:
        self._check("muon_polar_scratch_init", self.lib.muon_polar_scratch_init(
            scratch.data_ptr(), _nbytes(scratch), self._stream(stream)))

    def new_scratch(self, batch: int, m: int, n: int, device=None, stream=None):
        """A zero-initialised split-K scratch buffer (uint8 tensor, possibly
        empty) for problems of this size on the current device."""
        import torch

        nbytes = self.scratch_bytes(batch, m, n)
        scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device or "cuda")
        if nbytes:
            self.scratch_init(scratch, stream)
        return scratch

    # -------------------------------------------------------------- kernels
    # Tensors are torch tensors on the current CUDA device; x is [B, M, ld]
    # with the first n columns valid.  `scratch` (optional) enables split-K.
    def gram(self, x, gram, n: Optional[int] = None, scratch=None, stream=None) -> None:
        b, m, ld = x.shape
        n = ld if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_gram_sm100", self.lib.muon_polar_gram_sm100(
            x.data_ptr(), gram.data_ptr(), b, m, n, ld, sp, sb, self._stream(stream)))

    def gram_static_scratch(self, x, gram, n: Optional[int] = None, stream=None) -> None:
        """Kernel 1 with split-K scratch taken from the array built into the
        library (for callers that cannot allocate device memory)."""
        b, m, ld = x.shape
        n = ld if n is None else n
        self._check("muon_polar_gram_static_scratch_sm100",
                    self.lib.muon_polar_gram_static_scratch_sm100(
                        x.data_ptr(), gram.data_ptr(), b, m, n, ld, self._stream(stream)))

    def gram_f32(self, x, gram_f32, n: Optional[int] = None, scratch=None,
                 stream=None) -> None:
        b, m, ld = x.shape
        n = ld if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_gram_f32_sm100", self.lib.muon_polar_gram_f32_sm100(
            x.data_ptr(), gram_f32.data_ptr(), b, m, n, ld, sp, sb, self._stream(stream)))

    def gram_f32_band(self, x, gram_f32, row_begin: int, row_count: int, sm_reserve: int = 0,
                      n: Optional[int] = None, scratch=None, stream=None) -> None:
        """Upper tiles of rows [row_begin, row_begin + row_count) of the fp32
        Gram, mirrored; run band by band from row 0, each band's rows are
        complete once it has run."""
        b, m, ld = x.shape
        n = ld if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_gram_f32_band_sm100", self.lib.muon_polar_gram_f32_band_sm100(
            x.data_ptr(), gram_f32.data_ptr(), b, m, n, ld, int(row_begin), int(row_count),
            int(sm_reserve), sp, sb, self._stream(stream)))

    # Packed upper-triangle units ([B, units, 256, 256]) for column-sharded
    # callers: the rank's partial Gram is reduce-scattered by units.
    def packed_units(self, m: int) -> int:
        return int(self.lib.muon_polar_packed_units(int(m)))

    def gram_f32_packed(self, x, packed_f32, n: Optional[int] = None, scratch=None,
                        stream=None) -> None:
        b, m, ld = x.shape
        n = ld if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_gram_f32_packed_sm100",
                    self.lib.muon_polar_gram_f32_packed_sm100(
                        x.data_ptr(), packed_f32.data_ptr(), b, m, n, ld, sp, sb,
                        self._stream(stream)))

    def poly_packed(self, gram, packed_poly, b: float, c: float, unit_begin: int,
                    unit_count: int, stream=None) -> None:
        """Units [unit_begin, unit_begin + unit_count) of kernel (2)'s output
        into their places in the packed buffer, from the full bf16 gram."""
        bsz, mp, _ = gram.shape
        self._check("muon_polar_poly_packed_sm100", self.lib.muon_polar_poly_packed_sm100(
            gram.data_ptr(), packed_poly.data_ptr(), bsz, mp, int(unit_begin), int(unit_count),
            float(b), float(c), self._stream(stream)))

    def unpack_sym(self, packed, full, stream=None) -> None:
        """Packed bf16 units -> the full symmetric [B, Mp, Mp] bf16 matrix."""
        bsz, mp, _ = full.shape
        self._check("muon_polar_unpack_sym_sm100", self.lib.muon_polar_unpack_sym_sm100(
            packed.data_ptr(), full.data_ptr(), bsz, mp, self._stream(stream)))

    def poly(self, gram, poly, b: float, c: float, scratch=None, stream=None) -> None:
        bsz, mp, _ = gram.shape
        sp, sb = _scratch(scratch)
        self._check("muon_polar_poly_sm100", self.lib.muon_polar_poly_sm100(
            gram.data_ptr(), poly.data_ptr(), bsz, mp, float(b), float(c), sp, sb,
            self._stream(stream)))

    def poly_rows(self, gram, poly, b: float, c: float, row_begin: int, row_count: int,
                  stream=None) -> None:
        """Rows [row_begin, row_begin + row_count) of kernel (2)'s output,
        written into the full buffer `poly`."""
        bsz, mp, _ = gram.shape
        self._check("muon_polar_poly_rows_sm100", self.lib.muon_polar_poly_rows_sm100(
            gram.data_ptr(), poly.data_ptr(), bsz, mp, int(row_begin), int(row_count),
            float(b), float(c), self._stream(stream)))

    def apply(self, poly, x, y, a: float, n: Optional[int] = None, stream=None) -> None:
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        self._check("muon_polar_apply_sm100", self.lib.muon_polar_apply_sm100(
            poly.data_ptr(), x.data_ptr(), y.data_ptr(), bsz, m, n, ldx, y.shape[-1],
            float(a), self._stream(stream)))

    def step(self, x, y, workspace, a: float, b: float, c: float,
             n: Optional[int] = None, scratch=None, stream=None) -> None:
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_step_sm100", self.lib.muon_polar_step_sm100(
            x.data_ptr(), y.data_ptr(), workspace.data_ptr(), _nbytes(workspace), sp, sb,
            bsz, m, n, ldx, y.shape[-1], float(a), float(b), float(c),
            self._stream(stream)))

    # The step of X^T returned in X's layout (M > N without transposed
    # copies): gram is [B, Np, Np] with Np = padded_rows(n).
    def gram_t(self, x, gram, n: Optional[int] = None, scratch=None, stream=None) -> None:
        b, m, ld = x.shape
        n = ld if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_gram_t_sm100", self.lib.muon_polar_gram_t_sm100(
            x.data_ptr(), gram.data_ptr(), b, m, n, ld, sp, sb, self._stream(stream)))

    def apply_t(self, poly, x, y, a: float, n: Optional[int] = None, stream=None) -> None:
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        self._check("muon_polar_apply_t_sm100", self.lib.muon_polar_apply_t_sm100(
            poly.data_ptr(), x.data_ptr(), y.data_ptr(), bsz, m, n, ldx, y.shape[-1],
            float(a), self._stream(stream)))

    def step_t(self, x, y, workspace, a: float, b: float, c: float,
               n: Optional[int] = None, scratch=None, stream=None) -> None:
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        sp, sb = _scratch(scratch)
        self._check("muon_polar_step_t_sm100", self.lib.muon_polar_step_t_sm100(
            x.data_ptr(), y.data_ptr(), workspace.data_ptr(), _nbytes(workspace), sp, sb,
            bsz, m, n, ldx, y.shape[-1], float(a), float(b), float(c),
            self._stream(stream)))

    # The caller side of the step: several steps, normalisation, Muon update.
    @staticmethod
    def _coefficients(coefficients):
        flat = [float(v) for row in coefficients for v in row]
        return (ctypes.c_float * len(flat))(*flat), len(flat) // 3

    @staticmethod
    def _dtype_code(t) -> int:
        import torch

        if t.dtype == torch.float32:
            return 0
        if t.dtype == torch.bfloat16:
            return 1
        raise TypeError(f"unsupported dtype {t.dtype}")

    def steps(self, x, y, buf0, buf1, workspace, coefficients, n: Optional[int] = None,
              scratch=None, stream=None) -> None:
        """len(coefficients) Polar Express steps of bf16 x ([B, M, ld]) into y,
        the intermediate iterates in buf0 / buf1 ([B, M, ldb]; None for one
        step)."""
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        coeffs, steps = self._coefficients(coefficients)
        sp, sb = _scratch(scratch)
        b0 = 0 if buf0 is None else buf0.data_ptr()
        b1 = 0 if buf1 is None else buf1.data_ptr()
        ldb = 0 if buf0 is None else buf0.shape[-1]
        self._check("muon_polar_steps_sm100", self.lib.muon_polar_steps_sm100(
            x.data_ptr(), y.data_ptr(), b0, b1, ldb, workspace.data_ptr(), _nbytes(workspace),
            sp, sb, bsz, m, n, ldx, y.shape[-1], coeffs, steps, self._stream(stream)))

    def express_workspace_bytes(self, batch: int, m: int, n: int) -> int:
        return int(self.lib.muon_polar_express_workspace_bytes(int(batch), int(m), int(n)))

    def polar_express(self, x, y, workspace, coefficients, normalize: bool = True,
                      n: Optional[int] = None, scratch=None, stream=None) -> None:
        """y = the Polar Express steps of x ([B, M, ld], fp32 or bf16, first n
        columns valid), after x / (||x||_F * 1.01 + 1e-6) when `normalize`."""
        bsz, m, ldx = x.shape
        n = ldx if n is None else n
        coeffs, steps = self._coefficients(coefficients)
        sp, sb = _scratch(scratch)
        self._check("muon_polar_express_sm100", self.lib.muon_polar_express_sm100(
            x.data_ptr(), self._dtype_code(x), ldx, y.data_ptr(), y.shape[-1],
            workspace.data_ptr(), _nbytes(workspace), sp, sb, bsz, m, n, coeffs, steps,
            1 if normalize else 0, self._stream(stream)))

    def muon_update(self, param, grad, momentum, workspace, lr: float, momentum_coef: float,
                    nesterov: bool, weight_decay: float, scale: float, coefficients,
                    scratch=None, stream=None) -> None:
        """One Muon update of contiguous [B, M, N] param / grad / momentum
        (one dtype, fp32 or bf16), in place on param and momentum."""
        bsz, m, n = param.shape
        coeffs, steps = self._coefficients(coefficients)
        sp, sb = _scratch(scratch)
        self._check("muon_polar_update_sm100", self.lib.muon_polar_update_sm100(
            param.data_ptr(), grad.data_ptr(), momentum.data_ptr(), self._dtype_code(param),
            workspace.data_ptr(), _nbytes(workspace), sp, sb, bsz, m, n, float(lr),
            float(momentum_coef), 1 if nesterov else 0, float(weight_decay), float(scale),
            coeffs, steps, self._stream(stream)))

    def update_launch_count(self) -> int:
        return int(self.lib.muon_polar_update_launch_count())

    def cast_f32_bf16(self, src, dst, stream=None) -> None:
        self._check("muon_polar_cast_f32_bf16_sm100", self.lib.muon_polar_cast_f32_bf16_sm100(
            src.data_ptr(), dst.data_ptr(), src.numel(), self._stream(stream)))


_CAPI: Optional[CAPI] = None


def capi() -> CAPI:
    """Process-wide CAPI instance (the library is loaded once)."""
    global _CAPI
    if _CAPI is None:
        _CAPI = CAPI()
    return _CAPI
