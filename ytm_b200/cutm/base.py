"""BaseTM — the reference's cutm host engine API (Mayur1009/YTM
src/cutm/base.py:41-593) over the B200 engine.

Same constructor arguments and defaults (base.py:16-29, 60-74), the same
derived sizes (base.py:94-121), the same fit/score/encode/transform/getter and
state-dict surface, the same array layouts and dtypes on the way out.  What
changes underneath: no runtime nvcc (hyper-parameters are runtime values),
bit-sliced TA states on the device, a decision stream keyed on the sample
counter instead of per-thread curand states, optional mini-batches, and clause
sharding over the ranks of a torch.distributed process group.
"""
from __future__ import annotations

import os
from typing import TypedDict

import numpy as np
import torch
import torch.distributed as dist

from .. import _lib
from ..engine import CudaEngine


class BaseTMOptArgs(TypedDict, total=False):
    q: float
    patch_dim: tuple[int, int]
    number_of_ta_states: int
    max_included_literals: int | None
    append_negated: bool
    init_neg_weights: bool
    negative_polarity: bool
    encode_loc: bool
    coalesced: bool
    h: float | list[float]
    bias: bool
    seed: int | None
    block_size: int


class FitOptArgs(TypedDict, total=False):
    block_size: int
    true_mod: list[float] | np.ndarray
    false_mod: list[float] | np.ndarray
    clause_drop_p: float
    norm_true_update_prob: bool
    norm_false_update_prob: bool
    batch_size: int


def _as_u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=np.uint32)


class BaseTM:
    """Tsetlin Machine on B200 GPUs (one clause shard per process).

    Extra keyword arguments beyond the reference's: ``device`` (CUDA device of
    this process, default the current one), ``process_group`` (a
    torch.distributed group to shard clauses over; default the world group when
    torch.distributed is initialised, else none) and ``inference_sharding``
    ("samples": every rank holds a replica of all include masks and weights,
    gathered once after each change, and scores its slice of the samples;
    "clauses": every rank scores all samples on its clauses and the class sums
    are all-reduced) and ``rules`` ("cutm": the rules of src/cutm/cuda/kernel.cu;
    "pytm": the rule variants of the reference's numpy TM, src/pytm/base.py —
    feedback for the true class and ONE uniformly drawn other class per
    sample, true class first, and clauses without includes counted at
    prediction).
    """

    def __init__(self, number_of_clauses_per_class: int, T: int, s: float, dim: tuple[int, int, int],
                 n_classes: int, device=None, process_group=None, inference_sharding: str = "samples",
                 rules: str = "cutm", _engine_factory=None, **opt_args):
        self.init_args = {"number_of_clauses_per_class": number_of_clauses_per_class, "T": T, "s": s,
                          "dim": tuple(dim), "n_classes": n_classes}
        self.opt_args: BaseTMOptArgs = {  # base.py:60-74
            "q": opt_args.get("q", 1.0),
            "patch_dim": tuple(opt_args.get("patch_dim", (dim[0], dim[1]))),
            "number_of_ta_states": opt_args.get("number_of_ta_states", 256),
            "max_included_literals": opt_args.get("max_included_literals", None),
            "append_negated": opt_args.get("append_negated", True),
            "init_neg_weights": opt_args.get("init_neg_weights", True),
            "negative_polarity": opt_args.get("negative_polarity", True),
            "encode_loc": opt_args.get("encode_loc", True),
            "coalesced": opt_args.get("coalesced", True),
            "h": opt_args.get("h", 1.0),
            "bias": opt_args.get("bias", False),
            "seed": opt_args.get("seed", None),
            "block_size": opt_args.get("block_size", 128),
        }
        unknown = set(opt_args) - set(self.opt_args)
        if unknown:
            raise TypeError(f"unexpected keyword arguments: {sorted(unknown)}")
        if self.opt_args["bias"]:
            # The reference marks bias "Does not work" (base.py:27); its kernel
            # updates the shared bias from every clause thread without atomics.
            raise NotImplementedError("bias=True is not supported")

        self.number_of_clauses_per_class = number_of_clauses_per_class
        self.T = T
        self.s = s
        self.dim = tuple(dim)
        self.number_of_outputs = n_classes
        self.q = min(self.opt_args["q"], float(n_classes))  # base.py:81
        self.patch_dim = self.opt_args["patch_dim"]
        self.number_of_ta_states = self.opt_args["number_of_ta_states"]
        self.max_included_literals = self.opt_args["max_included_literals"]
        self.append_negated = self.opt_args["append_negated"]
        self.init_neg_weights = self.opt_args["init_neg_weights"]
        self.negative_clauses = self.opt_args["negative_polarity"]
        self.encode_loc = self.opt_args["encode_loc"]
        self.coalesced = self.opt_args["coalesced"]
        self.bias = self.opt_args["bias"]
        self.block_size = self.opt_args["block_size"]
        h = self.opt_args["h"]
        if isinstance(h, list):
            assert len(h) == n_classes, "If h is a list, it must have length equal to n_classes."
        self.h = np.asarray(h if isinstance(h, list) else [h] * n_classes, dtype=np.float64)
        if not hasattr(self, "min_y"):
            self.min_y = None
        if not hasattr(self, "max_y"):
            self.max_y = None

        # process group / shard
        self._pg = process_group
        if self._pg is None and dist.is_available() and dist.is_initialized():
            self._pg = dist.group.WORLD
        self.world = dist.get_world_size(self._pg) if self._pg is not None else 1
        self.rank = dist.get_rank(self._pg) if self._pg is not None else 0

        seed = self.opt_args["seed"]
        if seed is None:
            seed = int.from_bytes(os.urandom(8), "little") >> 1
            if self.world > 1:  # every shard must use the same decision key
                t = torch.tensor([seed], dtype=torch.int64, device=self._comm_device(device))
                dist.broadcast(t, src=dist.get_global_rank(self._pg, 0), group=self._pg)
                seed = int(t.item())
        self.seed = self.opt_args["seed"]
        self._key = int(seed)
        self.rng = np.random.default_rng(self.seed)  # host RNG, as base.py:123 (clause drop)

        full = _lib.make_config(
            clauses_per_class=number_of_clauses_per_class, T=T, s=s, dim=self.dim, n_classes=n_classes, q=self.q,
            patch_dim=self.patch_dim, number_of_ta_states=self.number_of_ta_states,
            max_included_literals=self.max_included_literals, append_negated=self.append_negated,
            init_neg_weights=self.init_neg_weights, negative_polarity=self.negative_clauses,
            encode_loc=self.encode_loc, coalesced=self.coalesced, seed=self._key,
            one_negative=rules == "pytm", count_empty=rules == "pytm")
        if rules not in ("cutm", "pytm"):
            raise ValueError("rules must be 'cutm' or 'pytm'")
        self.rules = rules
        self.cfg_full = full
        self.number_of_clause_banks = full.clause_banks
        self.number_of_clauses = full.clauses
        self.number_of_literals = full.literals
        self.number_of_literal_chunks = full.words
        self.number_of_patches = full.patches
        self.cfg = _lib.shard_config(full, self.rank, self.world) if self.world > 1 else full
        self.clause_lo, self.clause_count = self.cfg.clause_lo, self.cfg.clause_count
        factory = _engine_factory or CudaEngine
        self.engine = factory(self.cfg, device)
        self.device = self.engine.device
        self.sample_counter = 0  # global sample counter t of the decision stream
        if inference_sharding not in ("samples", "clauses"):
            raise ValueError("inference_sharding must be 'samples' or 'clauses'")
        self.inference_sharding = inference_sharding
        self._model_version = 0  # bumped by every change of states or weights
        self._replica = None     # (version, include masks, weights) for sample-sharded inference
        self.last_class_sums = None  # class sums (int32, device) of the last trained batch

    # -- process group helpers -------------------------------------------------
    def _comm_device(self, device=None):
        if self._pg is not None and dist.get_backend(self._pg) == "nccl":
            if device is not None:
                return torch.device(device)
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")

    def _nccl(self):
        """NCCL communicator of the clause shards for the C training loop
        (None for one process or a non-NCCL group).  Made on first use: rank
        0's id is broadcast through the process group."""
        if self.world == 1 or dist.get_backend(self._pg) != "nccl":
            return None
        if getattr(self, "_comm", None) is None:
            import ctypes as ct
            lib = _lib.load()
            idb = torch.zeros(128, dtype=torch.uint8)
            if self.rank == 0:
                _lib.check(lib.ytm_nccl_unique_id(ct.c_void_p(idb.data_ptr())), "ytm_nccl_unique_id")
            idd = idb.to(self.device)
            dist.broadcast(idd, src=dist.get_global_rank(self._pg, 0), group=self._pg)
            idb = idd.cpu()
            comm = ct.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(lib.ytm_nccl_comm_init(ct.c_void_p(idb.data_ptr()), self.rank, self.world, ct.byref(comm)),
                           "ytm_nccl_comm_init")
            self._comm = comm
        return self._comm

    # class sums above this many int32 values go through NCCL: measured on 2
    # B200s, 2,560 values (config 2) take 9.2 us by the peer kernel against
    # 23.5 us for NCCL, 102,400 values (config 5) 25.8 us against 18.2 us
    PEER_AR_MAX_VALUES = 16384

    def _peer_ar(self, n: int):
        """One-shot peer-memory all-reduce context for the C training loop
        (all ranks on one node, NCCL group, at most PEER_AR_MAX_VALUES values;
        YTM_ALLREDUCE=nccl opts out), or None.  Made on first use with room
        for n values."""
        if self.world == 1 or dist.get_backend(self._pg) != "nccl" or os.environ.get("YTM_ALLREDUCE") == "nccl" \
                or n > self.PEER_AR_MAX_VALUES:
            return None
        ctx = getattr(self, "_par", None)
        if ctx is not None and self._par_n >= n:
            return ctx
        import ctypes as ct
        import socket
        hosts = [None] * self.world
        dist.all_gather_object(hosts, socket.gethostname(), group=self._pg)
        if len(set(hosts)) != 1 or self.world > 8:
            return None
        lib = _lib.load()
        if ctx is not None:  # regrow: every rank is done with the old buffers once all are here
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self._pg)
            _lib.check(lib.ytm_peer_ar_destroy(ctx), "ytm_peer_ar_destroy")
            self._par = None
        n = max(n, 1 << 16)
        ctx = ct.c_void_p()
        h = (ct.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.ytm_peer_ar_create(self.rank, self.world, n, ct.byref(ctx), h), "ytm_peer_ar_create")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=self._pg)
        allh = (ct.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(handles))
        with torch.cuda.device(self.device):
            _lib.check(lib.ytm_peer_ar_open(ctx, allh), "ytm_peer_ar_open")
        dist.barrier(group=self._pg)
        self._par, self._par_n = ctx, n
        return ctx

    def _check_peer_status(self, ctx) -> None:
        """Raise if a peer all-reduce since the last check gave up waiting for
        a rank (its slices were then left partly summed, so the ranks' models
        have diverged).  Synchronises the device once."""
        import ctypes as ct
        st = ct.c_int32(0)
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().ytm_peer_ar_status(ctx, ct.byref(st)), "ytm_peer_ar_status")
        if st.value:
            raise _lib.YTMError(f"peer all-reduce: rank {st.value - 1} did not arrive in time; "
                                "the clause shards are no longer consistent")

    def close(self) -> None:
        """Release the multi-GPU resources (peer all-reduce buffers and their
        IPC mappings, the NCCL communicator).  Call on every rank, before
        destroy_process_group; the model stays usable on one process."""
        lib = _lib.load() if (getattr(self, "_par", None) is not None or getattr(self, "_comm", None) is not None) \
            else None
        if lib is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self._pg)
        if getattr(self, "_par", None) is not None:
            _lib.check(lib.ytm_peer_ar_destroy(self._par), "ytm_peer_ar_destroy")
            self._par = None
        if getattr(self, "_comm", None) is not None:
            _lib.check(lib.ytm_nccl_comm_destroy(self._comm), "ytm_nccl_comm_destroy")
            self._comm = None

    def _allreduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        if dist.get_backend(self._pg) == "nccl" or t.device.type == "cpu":
            dist.all_reduce(t, group=self._pg)
            return t
        h = t.cpu()
        dist.all_reduce(h, group=self._pg)
        return h.to(t.device)

    def _gather_clauses(self, a: np.ndarray) -> np.ndarray:
        """Concatenate shard-local rows (axis 0 = clauses) of every rank."""
        if self.world == 1:
            return a
        parts = [None] * self.world
        dist.all_gather_object(parts, a, group=self._pg)
        return np.concatenate(parts, axis=0)

    def _gather_clause_axis1(self, a: np.ndarray) -> np.ndarray:
        if self.world == 1:
            return a
        parts = [None] * self.world
        dist.all_gather_object(parts, a, group=self._pg)
        return np.concatenate(parts, axis=1)

    def _to_device(self, a, dtype=np.uint32) -> torch.Tensor:
        if isinstance(a, torch.Tensor):
            return a.to(self.device, dtype=torch.int32).contiguous()
        a = np.ascontiguousarray(np.asarray(a), dtype=dtype)
        return torch.from_numpy(a.view(np.int32)).to(self.device)

    # -- resets (base.py:208-222) ----------------------------------------------------
    def _reset_clauses(self):
        self._model_version += 1
        self.engine.reset_state()

    def _reset_weights(self, reset_bias: bool = True):
        self._model_version += 1
        self.engine.reset_weights()

    # -- encoding (base.py:224-263) ----------------------------------------------------
    def _host_rows_sharded(self, X) -> bool:
        """Host inputs on a multi-GPU NCCL group: each rank copies only its
        share of the rows and the encoded rows are all-gathered over NVLink."""
        on_host = not isinstance(X, torch.Tensor) or X.device.type == "cpu"
        return (on_host and self.world > 1 and self.device.type == "cuda" and X.shape[0] >= self.world
                and dist.get_backend(self._pg) == "nccl")

    def _sharded_input(self, X, fn) -> torch.Tensor:
        """fn(device rows) for all rows of host input X: rank r copies rows
        [r * n, (r + 1) * n) (n = ceil(N / world); the last share padded with
        zero rows), encodes them, and the encoded shares are all-gathered.
        Every rank ends with the same tensor as fn(all rows) gives, while the
        host-to-device traffic per rank is 1/world of the input."""
        N = X.shape[0]
        n = -(-N // self.world)
        lo, hi = min(N, self.rank * n), min(N, (self.rank + 1) * n)
        part = self._to_device(X[lo:hi])
        if hi - lo < n:
            part = torch.cat([part, part.new_zeros((n - (hi - lo),) + tuple(part.shape[1:]))])
        mine = fn(part).contiguous()
        full = torch.empty((n * self.world,) + tuple(mine.shape[1:]), dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(full, mine, group=self._pg)
        return full[:N]

    def _encode_device(self, X) -> torch.Tensor:
        if not isinstance(X, torch.Tensor):
            assert X.ndim == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
            assert X.dtype == np.uint32, "X must be of type np.uint32."
        if self._host_rows_sharded(X):
            assert X.shape[1] == self.dim[0] * self.dim[1] * self.dim[2], "X has the wrong number of features."
            return self._sharded_input(X, self.engine.encode)
        if isinstance(X, torch.Tensor):
            Xd = X.to(self.device).to(torch.int32).contiguous()
            assert Xd.dim() == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
        else:
            assert X.ndim == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
            assert X.dtype == np.uint32, "X must be of type np.uint32."
            Xd = self._to_device(X)
        assert Xd.shape[1] == self.dim[0] * self.dim[1] * self.dim[2], "X has the wrong number of features."
        return self.engine.encode(Xd)

    def _input_device(self, X) -> torch.Tensor:
        """Raw inputs -> the engine's input for training and inference:
        packed bit images [N, image_words] for convolutional models (patch
        literal words are then formed on the fly, never stored: P*W words per
        sample), per-patch literal words [N, 1, W] for single-patch models."""
        if self.number_of_patches == 1:
            return self._encode_device(X)
        if not isinstance(X, torch.Tensor):
            assert X.ndim == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
            assert X.dtype == np.uint32, "X must be of type np.uint32."
        if self._host_rows_sharded(X):
            assert X.shape[1] == self.dim[0] * self.dim[1] * self.dim[2], "X has the wrong number of features."
            return self._sharded_input(X, self.engine.pack_images)
        if isinstance(X, torch.Tensor):
            Xd = X.to(self.device).to(torch.int32).contiguous()
            assert Xd.dim() == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
        else:
            assert X.ndim == 2, "X must be a 2D array (samples, dim0 * dim1 * dim2)."
            assert X.dtype == np.uint32, "X must be of type np.uint32."
            Xd = self._to_device(X)
        assert Xd.shape[1] == self.dim[0] * self.dim[1] * self.dim[2], "X has the wrong number of features."
        return self.engine.pack_images(Xd)

    def encode(self, X, block_size: int | None = None) -> np.ndarray:
        """Raw u32 inputs [N, D0*D1*D2] -> encoded literals u32 [N, P, W] (host)."""
        return self._encode_device(X).cpu().numpy().view(np.uint32)

    def encode_thermometer(self, images, levels: int = 8, on_device: bool = False):
        """Thermometer-binarise and encode raw 8-bit images on the GPU.

        images: uint8 [N, H, W, C] or [N, H, W] (numpy or torch), with
        dim = (W, H, C * levels).  Same result as
        ``tm.encode(ThermometerBinarizer(levels).binarize_rgb(images).reshape(N, -1))``
        (tm_utils/binarizer.py:17-21) without the host's u32-per-bit array.
        Returns u32 [N, P, W] on the host, or the int32 device tensor with
        on_device=True (pass it to fit/predict with is_X_encoded=True)."""
        t = images if isinstance(images, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(images))
        if t.dtype != torch.uint8:
            raise TypeError("images must be uint8")
        t = t.reshape(t.shape[0], -1).to(self.device)
        if t.shape[1] * levels != self.dim[0] * self.dim[1] * self.dim[2]:
            raise ValueError("images do not match dim = (width, height, channels * levels)")
        lits = self.engine.encode_thermometer(t, levels)
        return lits if on_device else lits.cpu().numpy().view(np.uint32)

    def _literals_device(self, X, is_X_encoded: bool) -> torch.Tensor:
        if not is_X_encoded:
            return self._input_device(X)
        lits = self._to_device(X)
        return lits.reshape(-1, self.number_of_patches, self.number_of_literal_chunks)

    # -- fit (base.py:266-359) ---------------------------------------------------------
    def _fit(self, encoded_X, encoded_Y, **opt_args):
        batch_size = int(opt_args.get("batch_size", 1))
        clause_drop_p = opt_args.get("clause_drop_p", 0.0)
        # true_mod / false_mod / norm_*: accepted; the reference's
        # update_probability ignores them (kernel.cu:508-529).
        if batch_size < 1:
            raise ValueError("batch_size must be >= 1")
        lits = encoded_X if isinstance(encoded_X, torch.Tensor) and encoded_X.device == self.device \
            else self._literals_device(encoded_X, True)
        if not self._is_images(lits):
            lits = lits.reshape(-1, self.number_of_patches, self.number_of_literal_chunks)
        Y = self._to_device(encoded_Y, np.int32).reshape(-1, self.number_of_outputs)
        N = lits.shape[0]
        if clause_drop_p > 0.0:  # base.py:288-293: one mask per fit call, from the host RNG
            mask = (self.rng.random(self.number_of_clauses) <= clause_drop_p).astype(np.uint32)
        else:
            mask = None
        drop = None if mask is None else self._to_device(mask[self.clause_lo:self.clause_lo + self.clause_count])
        t = self.sample_counter
        self._model_version += 1
        if batch_size == 1 and self.world == 1 and N > 0 and self._fused_b1_ok() \
                and hasattr(self.engine, "train_fit_b1"):
            # the reference's per-sample loop, one fused launch per sample
            self.engine.train_fit_b1(lits, Y, t, drop)
            self.sample_counter = t + N
            self.last_class_sums = self.engine.b1_class_sums(N)
            return
        if hasattr(self.engine, "train_fit_batches") and (self.world == 1 or dist.get_backend(self._pg) == "nccl"):
            # the batch loop and the class-sum all-reduce queued from C
            par = self._peer_ar(min(batch_size, N) * self.number_of_outputs)
            self.last_class_sums = self.engine.train_fit_batches(lits, Y, batch_size, t, drop, self.rank == 0,
                                                                 None if par is not None else self._nccl(), par)
            self.sample_counter = t + N
            if par is not None:
                self._check_peer_status(par)
            return
        for i in range(0, N, batch_size):
            B = min(batch_size, N - i)
            lb, yb = lits[i:i + B], Y[i:i + B]
            cs = self.engine.train_eval(lb, t, drop, add_bias=self.rank == 0)
            cs = self._allreduce(cs)
            self.engine.train_update(cs, yb, lb, t, drop)
            t += B
            self.last_class_sums = cs
        self.sample_counter = t

    def _is_images(self, lits: torch.Tensor) -> bool:
        """Packed bit images (2-D) rather than per-patch literal words (3-D)."""
        return lits.dim() == 2 and self.number_of_patches > 1

    def _fused_b1_ok(self) -> bool:
        """Batch-1 training runs as one fused launch per sample unless the
        per-clause patch scan would be long (P * W above 16k words): then the
        tiled evaluation kernel of the general path is faster."""
        return self.number_of_patches * self.number_of_literal_chunks <= 16384

    # -- inference (base.py:375-420) --------------------------------------------------
    def _gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """Concatenate every rank's shard-local rows of t (clause axis 0)."""
        counts = [_lib.shard_config(self.cfg_full, r, self.world).clause_count for r in range(self.world)]
        m = max(counts)
        pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        pad[:t.shape[0]] = t
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=self._pg)
        return torch.cat([p[:n] for p, n in zip(parts, counts)]).contiguous()

    def _replicated_model(self):
        if self._replica is None or self._replica[0] != self._model_version:
            inc, _ = self.engine.include_mask()
            self._replica = (self._model_version, self._gather_rows(inc), self._gather_rows(self.engine.weights))
        return self._replica[1], self._replica[2]

    def _score_samples_sharded(self, lits: torch.Tensor) -> torch.Tensor:
        N = lits.shape[0]
        inc, w = self._replicated_model()
        per = -(-N // self.world)
        lo, hi = min(N, per * self.rank), min(N, per * (self.rank + 1))
        cs = torch.zeros((per, self.number_of_outputs), dtype=torch.int32, device=self.device)
        if hi > lo:
            cs[:hi - lo] = self.engine.infer_include(self.cfg_full, inc, w, lits[lo:hi], self.engine.bias)
        parts = [torch.empty_like(cs) for _ in range(self.world)]
        dist.all_gather(parts, cs, group=self._pg)
        return torch.cat(parts)[:N]

    def _score_device(self, lits: torch.Tensor, chunk: int | None = None) -> torch.Tensor:
        N = lits.shape[0]
        if self.world > 1 and self.inference_sharding == "samples":
            return self._score_samples_sharded(lits)
        if chunk is None:
            per = max(1, (lits.shape[1] if self._is_images(lits) else
                          self.number_of_patches * self.number_of_literal_chunks) * 4
                      + ((self.clause_count + 31) // 32) * 4)
            chunk = max(1, min(N, (1 << 31) // per))
        outs = []
        for i in range(0, N, chunk):
            cs = self.engine.infer(lits[i:i + chunk], add_bias=self.rank == 0)
            outs.append(self._allreduce(cs))
        return torch.cat(outs) if outs else torch.empty((0, self.number_of_outputs), dtype=torch.int32,
                                                       device=self.device)

    def _score_batch(self, encoded_X, block_size: int | None = None) -> np.ndarray:
        lits = self._literals_device(encoded_X, True)
        return self._score_device(lits).cpu().numpy().astype(np.float32)

    # -- getters (base.py:423-461) ---------------------------------------------------------
    def _bank_shape(self, a: np.ndarray, last: int) -> np.ndarray:
        if self.coalesced:
            return a.reshape((self.number_of_clauses, last))
        return a.reshape((self.number_of_clause_banks, self.number_of_clauses_per_class, last))

    def get_ta_state(self):
        return self._bank_shape(self._gather_clauses(self.engine.get_ta_state()), self.number_of_literals)

    def get_literals(self):
        return (self.get_ta_state() > (self.number_of_ta_states // 2)).astype(np.uint32)

    def get_weights(self):
        w = self._gather_clauses(self.engine.weights.cpu().numpy()).astype(np.float32)
        return self._bank_shape(w, self.number_of_outputs)

    def get_patch_weights(self):
        pw = self._gather_clauses(self.engine.patch_w.cpu().numpy())
        return self._bank_shape(pw, self.number_of_patches)

    def get_bias_weights(self):
        return self.engine.bias.cpu().numpy().astype(np.float32)

    # -- transforms (base.py:465-542) -------------------------------------------------
    def transform(self, X, is_X_encoded: bool = False, block_size: int | None = None):
        lits = self._literals_device(X, is_X_encoded)
        out = self.engine.transform(lits).cpu().numpy().view(np.uint32)
        return self._gather_clause_axis1(out)

    def transform_patchwise(self, X, is_X_encoded: bool = False, block_size: int | None = None):
        lits = self._literals_device(X, is_X_encoded)
        out = self.engine.transform_patchwise(lits).cpu().numpy().view(np.uint32)
        return self._gather_clause_axis1(out)

    # -- serialization (base.py:547-593) ------------------------------------------------
    def __getstate__(self):
        args = {**self.init_args, **self.opt_args}
        return {"args": args, "state": self.get_state_dict()}

    def __setstate__(self, state):
        self.__init__(**state["args"])
        self.load_state_dict(state)

    def get_state_dict(self):
        return {
            "ta_state": self.get_ta_state().reshape(-1).astype(np.uint32),
            "clause_weights": self.get_weights().reshape(-1).astype(np.float32),
            "patch_weights": self.get_patch_weights().reshape(-1).astype(np.int32),
            "min_y": self.min_y,
            "max_y": self.max_y,
            "sample_counter": self.sample_counter,
            "decision_key": self._key,
        }

    def load_state_dict(self, state):
        sd = state["state"]
        C, L, K, P = self.number_of_clauses, self.number_of_literals, self.number_of_outputs, self.number_of_patches
        lo, n = self.clause_lo, self.clause_count
        ta = np.asarray(sd["ta_state"], dtype=np.uint32).reshape(C, L)[lo:lo + n]
        w = np.asarray(sd["clause_weights"], dtype=np.float32).reshape(C, K)[lo:lo + n]
        if not np.all(w == np.round(w)):
            raise ValueError("clause weights must be whole numbers")
        pw = np.asarray(sd["patch_weights"], dtype=np.int32).reshape(C, P)[lo:lo + n]
        self.min_y, self.max_y = sd["min_y"], sd["max_y"]
        self._model_version += 1
        self.engine.set_ta_state(ta)
        self.engine.weights.copy_(torch.from_numpy(np.ascontiguousarray(w.astype(np.int32))))
        self.engine.patch_w.copy_(torch.from_numpy(np.ascontiguousarray(pw)))
        self.sample_counter = int(sd.get("sample_counter", 0))
        if sd.get("decision_key") is not None and int(sd["decision_key"]) != self._key:
            # a model saved with seed=None keeps drawing from its own stream
            self._key = int(sd["decision_key"])
            self.cfg_full.seed = self._key
            self.cfg.seed = self._key
            self.engine.cfg.seed = self._key
