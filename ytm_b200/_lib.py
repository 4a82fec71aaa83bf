"""ctypes binding of libytm.so (include/ytm.h).

The library is required: importing this module on a machine without the built
library raises immediately; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as ct
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libytm.so")

YTM_OK = 0
YTM_OP_ENCODE, YTM_OP_INFER, YTM_OP_TRANSFORM, YTM_OP_TRAIN, YTM_OP_TRAIN_B1, YTM_OP_ENCODE_THERMO = 1, 2, 3, 4, 5, 6
YTM_OP_TRAIN_LOOP = 7

# Every function include/ytm.h declares; tests check the library exports them.
EXPORTS = (
    "ytm_config_init", "ytm_config_shard", "ytm_workspace_bytes", "ytm_encode", "ytm_state_init",
    "ytm_state_from_u32", "ytm_state_to_u32", "ytm_include_mask", "ytm_weights_init", "ytm_infer",
    "ytm_transform", "ytm_transform_patchwise", "ytm_train_eval", "ytm_train_update",
    "ytm_train_selection", "ytm_last_error", "ytm_version", "ytm_infer_noalloc",
    "ytm_train_fit_b1", "ytm_infer_include", "ytm_train_update_counted", "ytm_pack_images",
    "ytm_pack_images_thermometer",
    "ytm_encode_thermometer", "ytm_nccl_unique_id", "ytm_nccl_comm_init", "ytm_nccl_comm_destroy",
    "ytm_train_fit_batches", "ytm_peer_ar_create", "ytm_peer_ar_open", "ytm_peer_allreduce_i32",
    "ytm_peer_ar_status", "ytm_peer_ar_destroy", "ytm_config_size", "ytm_match_counters",
)


class YTMError(RuntimeError):
    pass


class Config(ct.Structure):
    """Mirror of struct ytm_config."""
    _fields_ = [
        ("clauses_per_class", ct.c_int32), ("T", ct.c_int32), ("s", ct.c_double), ("q", ct.c_double),
        ("dim0", ct.c_int32), ("dim1", ct.c_int32), ("dim2", ct.c_int32), ("n_classes", ct.c_int32),
        ("patch_dim0", ct.c_int32), ("patch_dim1", ct.c_int32), ("number_of_ta_states", ct.c_int32),
        ("max_included_literals", ct.c_int32), ("append_negated", ct.c_int32),
        ("init_neg_weights", ct.c_int32), ("negative_polarity", ct.c_int32), ("encode_loc", ct.c_int32),
        ("coalesced", ct.c_int32), ("seed", ct.c_uint64),
        ("clause_banks", ct.c_int32), ("clauses", ct.c_int32), ("literals", ct.c_int32),
        ("words", ct.c_int32), ("patches", ct.c_int32), ("half_literals", ct.c_int32),
        ("loc_literals", ct.c_int32),
        ("max_state", ct.c_int32), ("half_state", ct.c_int32), ("planes", ct.c_int32),
        ("state_offset", ct.c_int32), ("state_top", ct.c_int32),
        ("s_count_cdf", ct.c_uint32 * 32), ("q_threshold", ct.c_uint64),
        ("q_count_cdf", ct.c_uint32 * 32), ("q_select", ct.c_int32),
        ("run_cdf16", (ct.c_uint32 * 65) * 8),
        ("clause_lo", ct.c_int32), ("clause_count", ct.c_int32),
        ("one_negative", ct.c_int32), ("count_empty", ct.c_int32),
        ("input_images", ct.c_int32), ("image_words", ct.c_int32),
        ("run_range", ct.c_uint32 * 8),
    ]


_P = ct.c_void_p
_I32, _I64, _U64 = ct.c_int32, ct.c_int64, ct.c_uint64
_CFG = ct.POINTER(Config)

_SIGS = {
    "ytm_config_init": ([_CFG, _I32, _I32, ct.c_double, _I32, _I32, _I32, _I32, ct.c_double, _I32, _I32, _I32,
                         _I32, _I32, _I32, _I32, _I32, _I32, _U64], ct.c_int),
    "ytm_config_shard": ([_CFG, _I32, _I32], ct.c_int),
    "ytm_workspace_bytes": ([_CFG, _I32, _I64], _U64),
    "ytm_encode": ([_CFG, _P, _I64, _P, _P, _P], ct.c_int),
    "ytm_state_init": ([_CFG, _P, _P], ct.c_int),
    "ytm_state_from_u32": ([_CFG, _P, _P, _P], ct.c_int),
    "ytm_state_to_u32": ([_CFG, _P, _P, _P], ct.c_int),
    "ytm_include_mask": ([_CFG, _P, _P, _P, _P], ct.c_int),
    "ytm_weights_init": ([_CFG, _P, _P], ct.c_int),
    "ytm_infer": ([_CFG, _P, _P, _P, _P, _I64, _P, _P, _P], ct.c_int),
    "ytm_transform": ([_CFG, _P, _P, _I64, _P, _P, _P], ct.c_int),
    "ytm_transform_patchwise": ([_CFG, _P, _P, _I64, _P, _P], ct.c_int),
    "ytm_train_eval": ([_CFG, _P, _P, _P, _P, _P, _I32, _U64, _I32, _P, _P, _P, _P], ct.c_int),
    "ytm_train_update": ([_CFG, _P, _P, _P, _P, _P, _P, _I32, _U64, _P, _P, _P, _P], ct.c_int),
    "ytm_pack_images": ([_CFG, _P, _I64, _P, _P], ct.c_int),
    "ytm_pack_images_thermometer": ([_CFG, _P, _I64, _I32, _P, _P], ct.c_int),
    "ytm_train_update_counted": ([_CFG, _P, _P, _P, _P, _P, _P, _I32, _U64, _P, _P, _P, _P, _P], ct.c_int),
    "ytm_train_selection": ([_CFG, _I32, _P, _P, _P], ct.c_int),
    "ytm_train_fit_b1": ([_CFG, _P, _P, _P, _P, _P, _P, _I64, _U64, _P, _P, _P], ct.c_int),
    "ytm_infer_noalloc": ([_CFG, _P, _P, _P, _P, _I64, _P, _P], ct.c_int),
    "ytm_match_counters": ([_P, _P], ct.c_int),
    "ytm_infer_include": ([_CFG, _P, _P, _P, _P, _I64, _P, _P, _P], ct.c_int),
    "ytm_encode_thermometer": ([_CFG, _P, _I64, _I32, _P, _P, _P], ct.c_int),
    "ytm_nccl_unique_id": ([_P], ct.c_int),
    "ytm_nccl_comm_init": ([_P, _I32, _I32, ct.POINTER(ct.c_void_p)], ct.c_int),
    "ytm_nccl_comm_destroy": ([_P], ct.c_int),
    "ytm_train_fit_batches": ([_CFG, _P, _P, _P, _P, _P, _P, _I64, _I32, _U64, _I32, _P, _P, _P, _P, _P], ct.c_int),
    "ytm_peer_ar_create": ([_I32, _I32, _I64, ct.POINTER(ct.c_void_p), _P], ct.c_int),
    "ytm_peer_ar_open": ([_P, _P], ct.c_int),
    "ytm_peer_allreduce_i32": ([_P, _P, _I64, _I64, _P], ct.c_int),
    "ytm_peer_ar_status": ([_P, ct.POINTER(ct.c_int32)], ct.c_int),
    "ytm_peer_ar_destroy": ([_P], ct.c_int),
    "ytm_last_error": ([], ct.c_char_p),
    "ytm_version": ([], ct.c_char_p),
    "ytm_config_size": ([], ct.c_int32),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load libytm.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise YTMError(f"{path} is missing: build it with `python -m ytm_b200.build` "
                       "(the engine has no CPU fallback)")
    lib = ct.CDLL(path)
    for name, (args, res) in _SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    if lib.ytm_config_size() != ct.sizeof(Config):
        raise YTMError(f"{path} was built with a different ytm_config ({lib.ytm_config_size()} bytes, binding "
                       f"{ct.sizeof(Config)}): rebuild it")
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc != YTM_OK:
        msg = load().ytm_last_error().decode(errors="replace")
        raise YTMError(f"{what}: status {rc}: {msg}" if what else f"status {rc}: {msg}")


def make_config(*, clauses_per_class, T, s, dim, n_classes, q=1.0, patch_dim=None, number_of_ta_states=256,
                max_included_literals=None, append_negated=True, init_neg_weights=True, negative_polarity=True,
                encode_loc=True, coalesced=True, seed=0, one_negative=False, count_empty=False) -> Config:
    if patch_dim is None:
        patch_dim = (dim[0], dim[1])
    cfg = Config()
    rc = load().ytm_config_init(
        ct.byref(cfg), int(clauses_per_class), int(T), float(s), int(dim[0]), int(dim[1]), int(dim[2]),
        int(n_classes), float(q), int(patch_dim[0]), int(patch_dim[1]), int(number_of_ta_states),
        -1 if max_included_literals is None else int(max_included_literals), int(bool(append_negated)),
        int(bool(init_neg_weights)), int(bool(negative_polarity)), int(bool(encode_loc)), int(bool(coalesced)),
        int(seed) & (2 ** 64 - 1))
    check(rc, "ytm_config_init")
    cfg.one_negative = int(bool(one_negative))
    cfg.count_empty = int(bool(count_empty))
    return cfg


def shard_config(cfg: Config, rank: int, world: int) -> Config:
    out = Config()
    ct.pointer(out)[0] = cfg
    check(load().ytm_config_shard(ct.byref(out), int(rank), int(world)), "ytm_config_shard")
    return out
