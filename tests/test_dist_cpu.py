"""Clause sharding over 2 gloo ranks on CPU: the host orchestration of
ytm_b200.cutm (shard ranges, seed broadcast, class-sum all-reduce, gathers of
states, weights and transforms) driven with a test-only engine that runs the
oracle on each rank's clause shard.  Results must equal one unsharded oracle
run."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

KW = dict(number_of_clauses_per_class=30, T=12, s=4.0, dim=(6, 6, 1), n_classes=3, patch_dim=(4, 4), seed=77)


class OracleShardEngine:
    """Same interface as ytm_b200.engine.CudaEngine, computed by the oracle on
    the CPU for the clause shard in cfg (test double)."""

    def __init__(self, cfg, device=None):
        self.cfg = cfg
        self.device = torch.device("cpu")
        self.o = O.Oracle(number_of_clauses_per_class=cfg.clauses_per_class, T=cfg.T, s=cfg.s,
                          dim=(cfg.dim0, cfg.dim1, cfg.dim2), n_classes=cfg.n_classes, q=cfg.q,
                          patch_dim=(cfg.patch_dim0, cfg.patch_dim1), seed=cfg.seed,
                          coalesced=bool(cfg.coalesced))
        self.lo, self.C = cfg.clause_lo, cfg.clause_count
        self.K, self.P, self.L = cfg.n_classes, cfg.patches, cfg.literals
        self._ta = np.zeros((self.C, self.L), np.uint32)
        self._w = np.zeros((self.C, self.K), np.int32)
        self._pw = np.zeros((self.C, self.P), np.int32)
        self.weights = torch.from_numpy(self._w)
        self.patch_w = torch.from_numpy(self._pw)
        self.bias = torch.zeros(self.K, dtype=torch.int32)
        self._last = None
        self.reset_state()
        self.reset_weights()

    def reset_state(self):
        self._ta[:] = self.o.init_state()[self.lo:self.lo + self.C]

    def reset_weights(self):
        self._w[:] = self.o.init_weights(self.lo, self.C)

    def _full_ta(self, others_zero=False):
        full = self.o.init_state()
        if others_zero:
            full[:] = 0
        full[self.lo:self.lo + self.C] = self._ta
        return full

    def include_mask(self):
        packed, ninc = self.o.pack(self._ta)
        return torch.from_numpy(packed.view(np.int32)), torch.from_numpy(ninc)

    def infer_include(self, cfg_full, inc, weights, lits, bias):
        # states with exactly these include bits: half+1 where included, 0 elsewhere
        bits = np.unpackbits(inc.numpy().view(np.uint32).view(np.uint8), axis=1, bitorder="little")[:, :self.L]
        ta = np.where(bits == 1, self.o.half_state + 1, 0).astype(np.uint32)
        return torch.from_numpy(self.o.infer(ta, weights.numpy(), self._lits(lits)))

    def encode(self, X):
        return torch.from_numpy(self.o.encode(X.numpy().view(np.uint32)).view(np.int32))

    def pack_images(self, X):  # the double keeps per-patch literal words
        return self.encode(X)

    def get_ta_state(self):
        return self._ta.copy()

    def set_ta_state(self, ta):
        self._ta[:] = ta

    @staticmethod
    def _lits(t):
        return t.numpy().view(np.uint32)

    def infer(self, lits, add_bias=True):
        full_w = np.zeros((self.o.C, self.K), np.int32)
        full_w[self.lo:self.lo + self.C] = self._w
        # clauses of other shards are empty (all states 0) and carry weight 0
        return torch.from_numpy(self.o.infer(self._full_ta(True), full_w, self._lits(lits)))

    def transform(self, lits):
        out = self.o.transform(self._full_ta(), self._lits(lits))[:, self.lo:self.lo + self.C]
        return torch.from_numpy(out.astype(np.int32))

    def transform_patchwise(self, lits):
        out = self.o.transform_patchwise(self._full_ta(), self._lits(lits))[:, self.lo:self.lo + self.C]
        return torch.from_numpy(out.astype(np.int32))

    def train_eval(self, lits_b, t0, drop, add_bias):
        lb = self._lits(lits_b)
        cs, sel, ninc = self.o.train_eval(self.lo, self._ta, self._w, lb, lb.shape[0], t0, patch_w=self._pw)
        self._last = (sel, ninc)
        return torch.from_numpy(cs)

    def train_update(self, cs, Y_b, lits_b, t0, drop, sel_override=None):
        sel, ninc = self._last
        lb = self._lits(lits_b)
        self.o.train_update(self.lo, self._ta, self._w, cs.numpy(), Y_b.numpy(), lb, lb.shape[0], t0, sel, ninc)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    rng = np.random.default_rng(0)
    X = (rng.random((24, 36)) < 0.4).astype(np.uint32)
    y = rng.integers(0, 3, 24)
    return X, y


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ytm_b200.cutm import MultiClassTM
        tm = MultiClassTM(_engine_factory=OracleShardEngine, **KW)
        assert tm.world == world and tm.clause_count < tm.number_of_clauses
        X, y = _data()
        tm.fit(X, y, batch_size=4)
        tm.fit(X, y, batch_size=4)
        ta, w, pw = tm.get_ta_state(), tm.get_weights(), tm.get_patch_weights()
        pred, cs = tm.predict(X)
        tm.inference_sharding = "clauses"
        pred2, cs2 = tm.predict(X)
        assert np.array_equal(cs, cs2)
        tr = tm.transform(X)
        if rank == 0:
            np.savez(os.path.join(out_dir, "dist.npz"), ta=ta, w=w, pw=pw, cs=cs, tr=tr, t=tm.sample_counter)
    finally:
        dist.destroy_process_group()


def test_two_rank_clause_sharding_matches_single_process(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got = np.load(tmp_path / "dist.npz")
    o = O.Oracle(**KW)
    X, y = _data()
    lits = o.encode(X)
    Y = O.encode_Y_multiclass(y, 3, KW["T"])
    ta, w, pw = o.init_state(), o.init_weights(), np.zeros((o.C, o.P), np.int32)
    t = o.fit(ta, w, pw, lits, Y, 0, batch_size=4)
    t = o.fit(ta, w, pw, lits, Y, t, batch_size=4)
    assert int(got["t"]) == t == 48
    np.testing.assert_array_equal(got["ta"], ta)
    np.testing.assert_array_equal(got["w"], w.astype(np.float32))
    np.testing.assert_array_equal(got["pw"], pw)
    np.testing.assert_array_equal(got["cs"], o.infer(ta, w, lits).astype(np.float32))
    np.testing.assert_array_equal(got["tr"], o.transform(ta, lits))
    assert not np.array_equal(ta, o.init_state())


def _seed_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ytm_b200.cutm import MultiClassTM
        kw = dict(KW)
        kw["seed"] = None
        tm = MultiClassTM(_engine_factory=OracleShardEngine, **kw)
        with open(os.path.join(out_dir, f"k{rank}"), "w") as f:
            f.write(str(tm._key))
    finally:
        dist.destroy_process_group()


def test_seed_none_is_shared_by_ranks(tmp_path):
    """With seed=None every rank must use rank 0's decision key."""
    mp.spawn(_seed_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    keys = [int(open(tmp_path / f"k{r}").read()) for r in range(2)]
    assert keys[0] == keys[1]


def _shard_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ytm_b200.cutm import MultiClassTM
        tm = MultiClassTM(_engine_factory=OracleShardEngine, **KW)
        X = np.arange(7 * 5, dtype=np.uint32).reshape(7, 5)
        calls = []

        def enc(t):  # stands in for the engine's encode: rows -> [rows, 2, 3]
            calls.append(t.shape[0])
            return (t[:, :3].unsqueeze(1).repeat(1, 2, 1) * 2 + 1).contiguous()
        res = {}
        for n in (7, 2, 3):  # shares 4+3 (last padded), 1+1, 2+1
            out = tm._sharded_input(X[:n], enc)
            res[f"n{n}"] = out.numpy()
            res[f"c{n}"] = np.array(calls[-1:])
        # host inputs on a gloo group are not sharded (the NCCL path only)
        res["sharded_on_gloo"] = np.array([tm._host_rows_sharded(X)])
        np.savez(os.path.join(out_dir, f"s{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def test_row_sharded_host_input_gathers_all_rows(tmp_path):
    """BaseTM._sharded_input on 2 gloo ranks: each rank encodes ceil(N/2)
    rows (the last share padded with zero rows) and every rank ends with the
    encoding of all N rows in order."""
    mp.spawn(_shard_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    X = np.arange(7 * 5, dtype=np.int32).reshape(7, 5)
    for r in range(2):
        got = np.load(tmp_path / f"s{r}.npz")
        for n in (7, 2, 3):
            want = np.repeat(X[:n, None, :3], 2, axis=1) * 2 + 1
            np.testing.assert_array_equal(got[f"n{n}"], want)
            assert got[f"c{n}"][0] == -(-n // 2)
        assert not got["sharded_on_gloo"][0]
