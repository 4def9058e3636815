"""ctypes binding of libneurogen_native.so (the B200 engine).

Same discovery contract as the reference adapter (neurogen/language/native.py:22-43):
``NEUROGEN_NATIVE_LIBRARY`` names an explicit library path; otherwise the in-tree build
``neurogen-2.5_b200/lib/libneurogen_native.so`` is used.  There is no fallback: a missing
library raises ``ValueError`` and a missing GPU makes ``ng_create`` fail with its error text.
"""
import ctypes as ct
import os
from pathlib import Path

import numpy as np

F32 = np.ctypeslib.ndpointer(dtype=np.float32, flags='C_CONTIGUOUS')
I32 = np.ctypeslib.ndpointer(dtype=np.int32, flags='C_CONTIGUOUS')
U32 = np.ctypeslib.ndpointer(dtype=np.uint32, flags='C_CONTIGUOUS')
I64 = np.ctypeslib.ndpointer(dtype=np.int64, flags='C_CONTIGUOUS')

PACKAGE_ROOT = Path(__file__).resolve().parents[1]
DEFAULT_LIBRARY = PACKAGE_ROOT / 'lib' / 'libneurogen_native.so'

# Every symbol the C header declares (include/neurogen_b200.h).
EXPORTS = (
    'ng_create', 'ng_destroy', 'ng_error', 'ng_backend', 'ng_step', 'ng_advance',
    'ng_state_size', 'ng_parameter_count', 'ng_step_batch', 'ng_advance_batch',
    'ng_pool_create', 'ng_pool_destroy', 'ng_pool_load', 'ng_pool_store', 'ng_pool_step',
    'ng_pool_step_device', 'ng_pool_device_state',
    'ng_net_default_config', 'ng_net_create', 'ng_net_create_edges', 'ng_net_destroy',
    'ng_net_synapses', 'ng_net_export', 'ng_net_set_state', 'ng_net_get_state', 'ng_net_run',
    'ng_net_run_device', 'ng_topology_create', 'ng_topology_destroy', 'ng_topology_synapses',
    'ng_topology_export', 'ng_net_create_topology', 'ng_net_stats', 'ng_step_static', 'ng_net_launch_kind',
    'ng_net_create_partitioned', 'ng_nccl_unique_id', 'ng_math_eval', 'ng_net_plasticity_state',
    'ng_net_exchange_kind',
)


class NetConfig(ct.Structure):
    """Mirror of ``ng_net_config`` (include/neurogen_b200.h)."""
    _fields_ = [
        ('n', ct.c_int32), ('n_exc', ct.c_int32), ('topology', ct.c_int32),
        ('p_connect', ct.c_float), ('fanin', ct.c_int32), ('bsr_blocks', ct.c_int32),
        ('bsr_fill', ct.c_int32), ('weight_kind', ct.c_int32), ('w_mu', ct.c_float),
        ('w_sigma', ct.c_float), ('delay_min', ct.c_int32), ('delay_max', ct.c_int32),
        ('seed', ct.c_uint64), ('dt_ms', ct.c_float), ('cap_exc_pf', ct.c_float),
        ('cap_inh_pf', ct.c_float), ('g_leak_ns', ct.c_float), ('e_leak_mv', ct.c_float),
        ('e_inh_mv', ct.c_float), ('v_thresh_mv', ct.c_float), ('v_reset_mv', ct.c_float),
        ('t_ref_ms', ct.c_float), ('tau_exc_ms', ct.c_float), ('tau_inh_ms', ct.c_float),
        ('tau_adapt_ms', ct.c_float), ('adapt_inc_pa', ct.c_float), ('bias_pa', ct.c_float),
        ('drive_kind', ct.c_int32), ('drive_p', ct.c_float), ('drive_ns', ct.c_float),
        ('storage', ct.c_int32), ('launch', ct.c_int32), ('part_rank', ct.c_int32),
        ('part_world', ct.c_int32), ('plasticity', ct.c_int32), ('stdp_rate', ct.c_float),
        ('inhibitory_rate', ct.c_float), ('target_hz', ct.c_float), ('scaling_tau_ms', ct.c_float),
        ('reserved', ct.c_int32 * 3),
    ]


_LIB = None


def library_path():
    explicit = os.environ.get('NEUROGEN_NATIVE_LIBRARY')
    return Path(explicit) if explicit else DEFAULT_LIBRARY


def library():
    """Load and type the engine library once per process."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.is_file():
        raise ValueError(f'B200 engine not built ({path}); run `make -C neurogen-2.5_b200` '
                         'or set NEUROGEN_NATIVE_LIBRARY')
    lib = ct.CDLL(str(path.resolve()))
    vp, sz, ci = ct.c_void_p, ct.c_size_t, ct.c_int
    lib.ng_create.argtypes = [ci] * 5 + [F32, sz, ct.c_char_p]
    lib.ng_create.restype = vp
    lib.ng_destroy.argtypes = [vp]
    lib.ng_destroy.restype = None
    lib.ng_error.argtypes = []
    lib.ng_error.restype = ct.c_char_p
    lib.ng_backend.argtypes = [vp]
    lib.ng_backend.restype = ct.c_char_p
    lib.ng_step.argtypes = [vp, ci, F32, sz, F32, F32, F32, F32]
    lib.ng_step.restype = ci
    lib.ng_advance.argtypes = [vp, F32, F32, sz, ci, F32, F32, F32]
    lib.ng_advance.restype = ci
    lib.ng_step_static.argtypes = [vp, ci, F32, sz, F32, F32, F32, F32]
    lib.ng_step_static.restype = ci
    lib.ng_math_eval.argtypes = [F32, sz, F32, F32]
    lib.ng_math_eval.restype = ci
    lib.ng_state_size.argtypes = [vp]
    lib.ng_state_size.restype = sz
    lib.ng_parameter_count.argtypes = [ci, ci, ci]
    lib.ng_parameter_count.restype = sz
    lib.ng_step_batch.argtypes = [vp, I32, ci, F32, sz, F32, F32, F32, F32]
    lib.ng_step_batch.restype = ci
    lib.ng_advance_batch.argtypes = [vp, F32, ci, F32, sz, ci, F32, F32, F32]
    lib.ng_advance_batch.restype = ci
    lib.ng_pool_create.argtypes = [vp, ci]
    lib.ng_pool_create.restype = vp
    lib.ng_pool_destroy.argtypes = [vp]
    lib.ng_pool_destroy.restype = None
    lib.ng_pool_load.argtypes = [vp, F32]
    lib.ng_pool_load.restype = ci
    lib.ng_pool_store.argtypes = [vp, F32]
    lib.ng_pool_store.restype = ci
    lib.ng_pool_step.argtypes = [vp, I32, vp, vp, vp]
    lib.ng_pool_step.restype = ci
    lib.ng_pool_step_device.argtypes = [vp, vp, vp, vp]
    lib.ng_pool_step_device.restype = ci
    lib.ng_pool_device_state.argtypes = [vp]
    lib.ng_pool_device_state.restype = vp
    cfgp = ct.POINTER(NetConfig)
    lib.ng_net_default_config.argtypes = [cfgp]
    lib.ng_net_default_config.restype = None
    lib.ng_net_create.argtypes = [cfgp]
    lib.ng_net_create.restype = vp
    lib.ng_net_create_edges.argtypes = [cfgp, ct.c_int64, I32, I32, I32, F32]
    lib.ng_net_create_edges.restype = vp
    lib.ng_net_destroy.argtypes = [vp]
    lib.ng_net_destroy.restype = None
    lib.ng_net_synapses.argtypes = [vp]
    lib.ng_net_synapses.restype = ct.c_int64
    lib.ng_net_launch_kind.argtypes = [vp]
    lib.ng_net_launch_kind.restype = ct.c_int
    lib.ng_net_export.argtypes = [vp, I32, I32, I32, F32]
    lib.ng_net_export.restype = ci
    lib.ng_net_set_state.argtypes = [vp, vp, vp, vp, vp, vp, vp, ct.c_int64]
    lib.ng_net_set_state.restype = ci
    lib.ng_net_get_state.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp]
    lib.ng_net_get_state.restype = ci
    lib.ng_net_run.argtypes = [vp, ci, vp, vp]
    lib.ng_net_run.restype = ci
    lib.ng_net_run_device.argtypes = [vp, ci, vp, vp, vp]
    lib.ng_net_run_device.restype = ci
    lib.ng_net_create_partitioned.argtypes = [cfgp, vp]
    lib.ng_net_create_partitioned.restype = vp
    lib.ng_nccl_unique_id.argtypes = [vp]
    lib.ng_nccl_unique_id.restype = ci
    lib.ng_net_stats.argtypes = [vp, I64]
    lib.ng_net_stats.restype = ci
    lib.ng_net_plasticity_state.argtypes = [vp, vp, vp, vp, vp, vp, vp]
    lib.ng_net_plasticity_state.restype = ci
    lib.ng_net_exchange_kind.argtypes = [vp]
    lib.ng_net_exchange_kind.restype = ci
    lib.ng_topology_create.argtypes = [cfgp]
    lib.ng_topology_create.restype = vp
    lib.ng_topology_destroy.argtypes = [vp]
    lib.ng_topology_destroy.restype = None
    lib.ng_topology_synapses.argtypes = [vp]
    lib.ng_topology_synapses.restype = ct.c_int64
    lib.ng_topology_export.argtypes = [vp, I32, I32, I32, F32]
    lib.ng_topology_export.restype = ci
    lib.ng_net_create_topology.argtypes = [vp]
    lib.ng_net_create_topology.restype = vp
    _LIB = lib
    return lib


def error():
    return library().ng_error().decode()


def ptr(array):
    """Raw address of a numpy array (or None)."""
    return None if array is None else array.ctypes.data_as(ct.c_void_p)
