"""ctypes backend module for the reference package (copy to src/refinekv/kernels/b200.py).

This is the binding a maintainer of Kevin-lkw/RefineKV-release would add to
keep the reference package and swap only its GPU backend for
librefinekv_b200.so.  The reference routes its GPU work through
``attention.py:_backend`` (``:17-40``) to ``select_blocks_triton``
(``kernels/runtime.py:93``) and ``sparse_attention_triton``
(``kernels/runtime.py:123``); ``build_summary`` (``summary.py:46``) is
torch-only.  The three functions below take the same arguments as those
and return the same results; ``_backend`` would return ``"b200"`` on sm_100
devices and call them.

The library is found as ``librefinekv_b200.so`` on the loader path, or at the
path in the RKV_LIBRARY environment variable.  Struct and argument types
follow include/refinekv_b200.h (ABI 2).
"""

import ctypes
import os

import torch

_lib = ctypes.CDLL(os.environ.get("RKV_LIBRARY", "librefinekv_b200.so"))


class _Summary(ctypes.Structure):  # struct rkv_summary
    _fields_ = [("key_pages", ctypes.c_void_p), ("value_pages", ctypes.c_void_p),
                ("key_page_head_stride", ctypes.c_int64), ("value_page_head_stride", ctypes.c_int64),
                ("counts", ctypes.c_void_p), ("key_mean", ctypes.c_void_p),
                ("value_mean", ctypes.c_void_p), ("ellipsoid", ctypes.c_void_p),
                ("value_norm", ctypes.c_void_p), ("max_value_norm", ctypes.c_void_p),
                ("heads", ctypes.c_int64), ("blocks", ctypes.c_int64), ("block_size", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("prompt_length", ctypes.c_int64),
                ("sequences", ctypes.c_int64), ("prompt_lengths", ctypes.c_void_p),
                ("page_table", ctypes.c_void_p), ("page_table_stride", ctypes.c_int64),
                ("pool_pages", ctypes.c_int64), ("key_page_stride", ctypes.c_int64),
                ("value_page_stride", ctypes.c_int64), ("key_token_stride", ctypes.c_int64),
                ("value_token_stride", ctypes.c_int64)]


_P = ctypes.c_void_p
_I = ctypes.c_int64
_lib.rkv_abi_version.restype = ctypes.c_int
_lib.rkv_last_error.restype = ctypes.c_char_p
_lib.rkv_decode_workspace_size.restype = ctypes.c_size_t
_lib.rkv_decode_workspace_size.argtypes = [_I, _I, _I, _I, _I]
_lib.rkv_select_workspace_size.restype = ctypes.c_size_t
_lib.rkv_select_workspace_size.argtypes = [_I, _I, _I, _I, _I]
for _name in ("rkv_summarize", "rkv_summarize_f32"):
    getattr(_lib, _name).argtypes = [_P, _P] + [_I] * 8 + [_P] * 9
_lib.rkv_select.argtypes = [ctypes.POINTER(_Summary), _P, ctypes.c_int, _I, _I, ctypes.c_float,
                            ctypes.c_int, _P, ctypes.c_int, _P, ctypes.c_size_t, _P]
_lib.rkv_decode.argtypes = [ctypes.POINTER(_Summary), _P, ctypes.c_int, _I, _P, _P, _I, _I, _I,
                            _I, _I, _P, _I, _P, ctypes.c_float, ctypes.c_int, _P, _P, _P,
                            ctypes.c_size_t, ctypes.c_uint, _P]
assert _lib.rkv_abi_version() == 2

_RED = {"mean": 0, "max": 1, "any": 2}
_PHASE_ALL = 15


def _check(rc):
    if rc:
        raise RuntimeError(_lib.rkv_last_error().decode())


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _view(s):  # BlockSummary -> rkv_summary (one prompt in its own pages)
    return _Summary(s.keys.data_ptr(), s.values.data_ptr(), s.keys.stride(0), s.values.stride(0),
                    s.counts.data_ptr(), s.key_mean.data_ptr(), s.value_mean.data_ptr(),
                    s.ellipsoid.data_ptr(), s.value_norm.data_ptr(), s.max_value_norm.data_ptr(),
                    s.keys.shape[0], s.counts.numel(), s.block_size, s.keys.shape[-1],
                    s.prompt_length, 1, None, None, 0, 0, 0, 0, 0, 0)


def _scratch(workspace, name, nbytes, device):  # the C ABI's workspace: zeroed once, reused
    t = workspace.get(name) if workspace is not None else None
    if t is None or t.numel() < nbytes:
        t = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        if workspace is not None:
            workspace[name] = t
    return t


def build_summary_b200(keys, values, block_size, summary_cls):
    """``summary.py:46`` on the GPU: bf16 or fp32 (heads, tokens, dim) caches.

    Pages are always a bf16 copy here for brevity (the mirror package's
    ``build_summary`` aliases a page-aligned bf16 cache instead).
    """
    heads, tokens, dim = keys.shape
    blocks = -(-tokens // block_size)
    dev = keys.device
    kp = torch.empty(heads, blocks, block_size, dim, dtype=torch.bfloat16, device=dev)
    vp = torch.empty_like(kp)
    km, vm, ell = (torch.empty(heads, blocks, dim, dtype=torch.bfloat16, device=dev)
                   for _ in range(3))
    vnorm = torch.empty(heads, blocks, dtype=torch.float32, device=dev)
    vmax = torch.empty(heads, dtype=torch.float32, device=dev)
    counts = torch.empty(blocks, dtype=torch.int64, device=dev)
    fn = _lib.rkv_summarize_f32 if keys.dtype == torch.float32 else _lib.rkv_summarize
    _check(fn(keys.data_ptr(), values.data_ptr(), heads, tokens, dim, keys.stride(0),
              keys.stride(1), values.stride(0), values.stride(1), block_size, kp.data_ptr(),
              vp.data_ptr(), km.data_ptr(), vm.data_ptr(), ell.data_ptr(), vnorm.data_ptr(),
              vmax.data_ptr(), counts.data_ptr(), _stream()))
    return summary_cls(kp, vp, counts, km, vm, ell, vnorm, vmax, tokens, block_size)


def select_blocks_b200(query, summary, config, workspace):
    """``runtime.py:93``: (H, G, 1, D) query -> bool (H, blocks) mask."""
    H, G, _, D = query.shape
    q = query.reshape(1, H, G, D).contiguous()
    mask = torch.empty(H, summary.num_blocks, dtype=torch.uint8, device=q.device)
    n = _lib.rkv_select_workspace_size(H, G, summary.num_blocks, D, 1)
    ws = _scratch(workspace, "b200_select", n, q.device)
    _check(_lib.rkv_select(ctypes.byref(_view(summary)), q.data_ptr(),
                           1 if q.dtype == torch.float32 else 0, 1, G, config.eps,
                           _RED[config.gqa_reduction], mask.data_ptr(), 0, ws.data_ptr(),
                           ws.numel(), _stream()))
    return mask.bool()


def sparse_attention_b200(query, summary, key_suffix, value_suffix, config, anchor_mask,
                          workspace, return_selected, suffix_length=None):
    """``runtime.py:123``: output (H, G, 1, D) in the query dtype and the optional mask."""
    H, G, _, D = query.shape
    q = query.reshape(H, G, D).contiguous()
    if key_suffix.dtype != torch.bfloat16:  # the reference rounds the suffix to bf16 too
        key_suffix, value_suffix = key_suffix.bfloat16(), value_suffix.bfloat16()
    out = torch.empty_like(q)
    sel = torch.empty(H, summary.num_blocks, dtype=torch.uint8, device=q.device)
    n = _lib.rkv_decode_workspace_size(H, G, summary.num_blocks, D, summary.block_size)
    ws = _scratch(workspace, "b200_decode", n, q.device)
    cap = key_suffix.shape[1]
    _check(_lib.rkv_decode(ctypes.byref(_view(summary)), q.data_ptr(),
                           1 if q.dtype == torch.float32 else 0, G,
                           key_suffix.data_ptr() if cap else None,
                           value_suffix.data_ptr() if cap else None, cap,
                           key_suffix.stride(0), key_suffix.stride(1),
                           value_suffix.stride(0), value_suffix.stride(1),
                           suffix_length.data_ptr() if suffix_length is not None else None, cap,
                           anchor_mask.data_ptr() if anchor_mask is not None else None,
                           config.eps, _RED[config.gqa_reduction], out.data_ptr(),
                           sel.data_ptr(), ws.data_ptr(), ws.numel(), _PHASE_ALL, _stream()))
    return out.view(H, G, 1, D), sel.bool() if return_selected else None
