"""ctypes binding of ``libflashns_b200.so`` (the C ABI in ``include/flashns_b200.h``).

There is no CPU or library fallback: every entry point needs the in-tree CUDA
library, and loading fails loudly when it has not been built.
"""

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libflashns_b200.so"

_c_int, _c_i64, _c_dbl, _c_ptr, _c_size = ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_void_p, ctypes.c_size_t

# name -> (argtypes); every function returns int (a cudaError_t value)
SIGNATURES = {
    "flashns_b200_plan_create": [_c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_int), _c_i64, _c_i64,
                                 _c_dbl, _c_dbl, _c_dbl, ctypes.POINTER(_c_ptr)],
    "flashns_b200_plan_destroy": [_c_ptr],
    "flashns_b200_plan_workspace_bytes": [_c_ptr, ctypes.POINTER(_c_size)],
    "flashns_b200_plan_parameter_count": [_c_ptr, ctypes.POINTER(_c_i64)],
    "flashns_b200_plan_launch_count": [_c_ptr, ctypes.POINTER(_c_int)],
    "flashns_b200_device_fault": [ctypes.POINTER(_c_int), _c_int],
    "flashns_b200_wait_selftest": [ctypes.c_uint, _c_ptr, _c_ptr],
    "flashns_b200_eval": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr],
    "flashns_b200_eval_marked": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr,
                                 _c_ptr, _c_int, ctypes.POINTER(_c_int)],
    "flashns_b200_plan_launch_kinds": [_c_ptr, ctypes.POINTER(_c_int), _c_int, ctypes.POINTER(_c_int)],
    "flashns_b200_fp64_peak_probe": [_c_int, _c_int, _c_ptr, ctypes.POINTER(_c_dbl), _c_ptr],
    "flashns_b200_fp64_probe": [_c_int, _c_int, _c_int, _c_int, _c_ptr, ctypes.POINTER(_c_dbl), _c_ptr],
    "flashns_b200_eval_static": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr],
    "flashns_b200_fields": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr],
    "flashns_b200_row_dots": [_c_ptr, _c_i64, _c_int, _c_ptr, _c_ptr, _c_i64, _c_ptr],
    "flashns_b200_lbfgs_pair_slot": [_c_ptr] * 6 + [_c_i64, _c_ptr, _c_i64, _c_ptr],
    "flashns_b200_lbfgs_ring_dots": [_c_ptr, _c_ptr, _c_i64, _c_int, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_i64, _c_ptr],
    "flashns_b200_lbfgs_commit": [_c_ptr, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr],
    "flashns_b200_lbfgs_coefficients": [_c_ptr, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr],
    "flashns_b200_lbfgs_direction": [_c_ptr, _c_ptr, _c_i64] + [_c_ptr] * 6 + [_c_i64, _c_ptr],
    "flashns_b200_lbfgs_save": [_c_ptr] * 6 + [_c_i64, _c_ptr],
    "flashns_b200_lbfgs_step_point": [_c_ptr] * 4 + [_c_i64, _c_ptr],
    "flashns_b200_adam_step": [_c_ptr] * 4 + [_c_i64, _c_dbl, _c_dbl, _c_dbl, _c_dbl, _c_i64, _c_ptr],
    "flashns_b200_residuals": [_c_int, _c_int, _c_ptr, _c_dbl, _c_ptr, _c_i64, _c_ptr],
    "flashns_b200_sobol_points": [_c_ptr, _c_ptr, _c_int, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_ptr],
    "flashns_b200_philox_points": [ctypes.c_uint64, ctypes.c_uint64, _c_int, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr,
                                   _c_i64, _c_ptr],
    "flashns_b200_pack_coordinates": [_c_ptr, _c_i64, _c_i64, _c_int, _c_ptr, _c_ptr],
    # reference-ABI hooks (experiments/pinn_v8/native.py:26-51, experiments/cuda_jet_h100/gpu.py)
    "flashns_v8_activation": [_c_int, _c_int] + [_c_ptr] * 5 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_coordinate_affine": [_c_int] + [_c_ptr] * 4 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_coordinate_affine_activation": [_c_int] + [_c_ptr] * 5 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_tail3": [_c_int, _c_int] + [_c_ptr] * 5 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_coordinate_wgrad": [_c_int] + [_c_ptr] * 5 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_coordinate_activation_wgrad": [_c_int] + [_c_ptr] * 7 + [_c_i64, _c_i64, _c_int, _c_ptr],
    "flashns_v8_loss_seed": [_c_ptr] * 8 + [_c_i64] * 3 + [_c_dbl] * 3 + [_c_ptr],
    "flashns_stable_activation": [_c_int, ctypes.c_bool] + [_c_ptr] * 5 + [_c_size, _c_size, _c_ptr],
    "flashns_stable_tail3": [_c_int, ctypes.c_bool] + [_c_ptr] * 5 + [_c_size, _c_size, _c_ptr],
    "flashns_stable_dgrad_vjp": [_c_int, ctypes.c_bool] + [_c_ptr] * 5 + [_c_int] * 3 + [_c_ptr],
    "flashns_stable_dgrad_shared_bytes": [],
    # the reference's Hopper plan names (experiments/cuda_jet_hopper/hopper.py:37-63)
    "flashns_hopper_initialize": [],
    "flashns_hopper_resources": [_c_int, ctypes.c_bool, ctypes.POINTER(ctypes.c_longlong)],
    "flashns_hopper_create": [_c_int, _c_ptr, _c_ptr, _c_int, _c_int, _c_int, ctypes.POINTER(_c_ptr)],
    "flashns_hopper_launch": [_c_ptr, _c_int, ctypes.c_bool, _c_ptr, _c_ptr, _c_ptr, _c_ptr],
}

KERNEL_KINDS = {0: "pack", 1: "first", 2: "forward", 3: "head", 4: "backward", 5: "wgrad", 6: "reduce",
                7: "forward_head"}

_library = None


def library():
    """Load the CUDA library once; raise if it is missing."""
    global _library
    if _library is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is missing: build it with `python -m flashns_b200.build` "
                               "(there is no CPU fallback)")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.flashns_hopper_destroy.argtypes = [_c_ptr]  # void, as the reference declares it
        lib.flashns_hopper_destroy.restype = None
        _library = lib
    return _library


def check(status, what):
    if status:
        raise RuntimeError(f"{what} returned CUDA error {status}")
