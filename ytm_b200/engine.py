"""Device-side engine of one clause shard: owns the shard's buffers (torch CUDA
tensors used as plain device memory) and drives libytm through its C ABI.

Buffers (C = clauses of the shard):
  state    bit-sliced TA states, u32 [planes][C][W]
  weights  i32 [C][K]
  patch_w  i32 [C][P]
  bias     i32 [K]
u32 data live in int32 tensors (same bytes); numpy views reinterpret them.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np
import torch

from . import _lib
from ._lib import check


def _p(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


class CudaEngine:
    """One clause shard on one CUDA device."""

    def __init__(self, cfg: _lib.Config, device: torch.device | str | int | None = None):
        self.lib = _lib.load()
        if not torch.cuda.is_available():
            raise _lib.YTMError("no CUDA device: the engine runs on B200 GPUs only (no CPU fallback)")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise _lib.YTMError(f"engine device must be CUDA, got {self.device}")
        self.cfg = cfg
        self.C, self.K, self.W, self.P = cfg.clause_count, cfg.n_classes, cfg.words, cfg.patches
        self.L, self.NB = cfg.literals, cfg.planes
        dev = self.device
        self.state = torch.empty(self.NB * self.C * self.W, dtype=torch.int32, device=dev)
        self.weights = torch.empty((self.C, self.K), dtype=torch.int32, device=dev)
        self.patch_w = torch.zeros((self.C, self.P), dtype=torch.int32, device=dev)
        self.bias = torch.zeros(self.K, dtype=torch.int32, device=dev)
        self._ws: dict[int, torch.Tensor] = {}
        self.reset_state()
        self.reset_weights()

    # -- plumbing -------------------------------------------------------------
    @property
    def _cfg(self):
        return ct.byref(self.cfg)

    @property
    def cfg_img(self) -> _lib.Config:
        """A copy of cfg for packed bit-image input (input_images = 1)."""
        c = _lib.Config.from_buffer_copy(self.cfg)
        c.input_images = 1 if self.P > 1 else 0
        return c

    def _cfg_for(self, lits: torch.Tensor | None):
        """The config matching the input form of `lits`: 2-D [N, image_words]
        tensors are packed bit images (convolutional models: input_images = 1),
        3-D [N, P, W] tensors per-patch literal words."""
        if lits is not None and lits.dim() == 2 and self.P > 1:
            return ct.byref(self.cfg_img)
        return self._cfg

    def _stream(self):
        return ct.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def workspace(self, op: int, n: int, cfg=None) -> torch.Tensor:
        need = int(self.lib.ytm_workspace_bytes(cfg if cfg is not None else self._cfg, op, int(n)))
        ws = self._ws.get(op)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
            self._ws[op] = ws
        return ws

    # -- state ------------------------------------------------------------------
    def reset_state(self):
        with torch.cuda.device(self.device):
            check(self.lib.ytm_state_init(self._cfg, _p(self.state), self._stream()), "ytm_state_init")

    def reset_weights(self):
        with torch.cuda.device(self.device):
            check(self.lib.ytm_weights_init(self._cfg, _p(self.weights), self._stream()), "ytm_weights_init")
        self.bias.zero_()

    def get_ta_state(self) -> np.ndarray:
        out = torch.empty((self.C, self.L), dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_state_to_u32(self._cfg, _p(self.state), _p(out), self._stream()), "ytm_state_to_u32")
        return out.cpu().numpy().view(np.uint32)

    def set_ta_state(self, ta: np.ndarray) -> None:
        ta = np.ascontiguousarray(np.asarray(ta, dtype=np.uint32).reshape(self.C, self.L))
        if ta.size and int(ta.max()) > self.cfg.state_top:
            raise ValueError(f"TA state {int(ta.max())} exceeds the representable maximum {self.cfg.state_top}")
        src = torch.from_numpy(ta.view(np.int32)).to(self.device)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_state_from_u32(self._cfg, _p(src), _p(self.state), self._stream()),
                  "ytm_state_from_u32")
        torch.cuda.current_stream(self.device).synchronize()

    def include_mask(self):
        inc = torch.empty((self.C, self.W), dtype=torch.int32, device=self.device)
        ninc = torch.empty(self.C, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_include_mask(self._cfg, _p(self.state), _p(inc), _p(ninc), self._stream()),
                  "ytm_include_mask")
        return inc, ninc

    # -- data path ----------------------------------------------------------------
    def encode(self, X: torch.Tensor) -> torch.Tensor:
        """X int32/uint32 [N, D] on this device -> literals int32 [N, P, W]."""
        X = X.contiguous()
        N = X.shape[0]
        lits = torch.empty((N, self.P, self.W), dtype=torch.int32, device=self.device)
        if N == 0:
            return lits
        ws = self.workspace(_lib.YTM_OP_ENCODE, N)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_encode(self._cfg, _p(X), N, _p(lits), _p(ws), self._stream()), "ytm_encode")
        return lits

    def pack_images(self, X: torch.Tensor) -> torch.Tensor:
        """X int32/uint32 [N, D] on this device -> packed bit images int32
        [N, image_words], the input form that forms patch literal words on the
        fly (models with several patches)."""
        X = X.contiguous()
        N = X.shape[0]
        out = torch.empty((N, self.cfg.image_words), dtype=torch.int32, device=self.device)
        if N:
            with torch.cuda.device(self.device):
                check(self.lib.ytm_pack_images(ct.byref(self.cfg_img), _p(X), N, _p(out), self._stream()),
                      "ytm_pack_images")
        return out

    def pack_images_thermometer(self, img: torch.Tensor, levels: int) -> torch.Tensor:
        """Raw uint8 images [N, dim0*dim1*channels] -> thermometer-binarised
        packed bit images int32 [N, image_words]."""
        img = img.contiguous()
        N = img.shape[0]
        out = torch.empty((N, self.cfg.image_words), dtype=torch.int32, device=self.device)
        if N:
            with torch.cuda.device(self.device):
                check(self.lib.ytm_pack_images_thermometer(ct.byref(self.cfg_img), _p(img), N, int(levels), _p(out),
                                                           self._stream()), "ytm_pack_images_thermometer")
        return out

    def encode_thermometer(self, img: torch.Tensor, levels: int) -> torch.Tensor:
        """Raw uint8 images [N, dim0*dim1*channels] on this device ->
        literals int32 [N, P, W] (thermometer binarisation on the device)."""
        img = img.contiguous()
        N = img.shape[0]
        lits = torch.empty((N, self.P, self.W), dtype=torch.int32, device=self.device)
        if N == 0:
            return lits
        ws = self.workspace(_lib.YTM_OP_ENCODE_THERMO, N)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_encode_thermometer(self._cfg, _p(img), N, int(levels), _p(lits), _p(ws),
                                                  self._stream()), "ytm_encode_thermometer")
        return lits

    def infer(self, lits: torch.Tensor, add_bias: bool = True) -> torch.Tensor:
        c = self._cfg_for(lits)
        N = lits.shape[0]
        cs = torch.empty((N, self.K), dtype=torch.int32, device=self.device)
        if N == 0:
            return cs
        ws = self.workspace(_lib.YTM_OP_INFER, N, c)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_infer(c, _p(self.state), _p(self.weights), _p(self.bias) if add_bias else None,
                                     _p(lits), N, _p(cs), _p(ws), self._stream()), "ytm_infer")
        return cs

    def infer_include(self, cfg_full: _lib.Config, inc: torch.Tensor, weights: torch.Tensor, lits: torch.Tensor,
                      bias: torch.Tensor | None) -> torch.Tensor:
        """Class sums from replicated include masks [C][W] and weights [C][K]
        of the whole model (cfg_full), for the given samples."""
        N = lits.shape[0]
        cs = torch.empty((N, self.K), dtype=torch.int32, device=self.device)
        if N == 0:
            return cs
        if lits.dim() == 2 and cfg_full.patches > 1:  # bit images
            cfg_full = _lib.Config.from_buffer_copy(cfg_full)
            cfg_full.input_images = 1
        need = int(self.lib.ytm_workspace_bytes(ct.byref(cfg_full), _lib.YTM_OP_INFER, N))
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_infer_include(ct.byref(cfg_full), _p(inc), _p(weights), _p(bias), _p(lits), N, _p(cs),
                                             _p(ws), self._stream()), "ytm_infer_include")
        return cs

    def transform(self, lits: torch.Tensor) -> torch.Tensor:
        c = self._cfg_for(lits)
        N = lits.shape[0]
        out = torch.empty((N, self.C), dtype=torch.int32, device=self.device)
        if N == 0:
            return out
        ws = self.workspace(_lib.YTM_OP_TRANSFORM, N, c)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_transform(c, _p(self.state), _p(lits), N, _p(out), _p(ws), self._stream()),
                  "ytm_transform")
        return out

    def transform_patchwise(self, lits: torch.Tensor) -> torch.Tensor:
        c = self._cfg_for(lits)
        N = lits.shape[0]
        out = torch.empty((N, self.C, self.P), dtype=torch.int32, device=self.device)
        if N == 0:
            return out
        with torch.cuda.device(self.device):
            check(self.lib.ytm_transform_patchwise(c, _p(self.state), _p(lits), N, _p(out), self._stream()),
                  "ytm_transform_patchwise")
        return out

    def train_eval(self, lits_b: torch.Tensor, t0: int, drop: torch.Tensor | None, add_bias: bool) -> torch.Tensor:
        c = self._cfg_for(lits_b)
        B = lits_b.shape[0]
        cs = torch.empty((B, self.K), dtype=torch.int32, device=self.device)
        ws = self.workspace(_lib.YTM_OP_TRAIN, B, c)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_train_eval(c, _p(self.state), _p(self.weights), _p(self.bias), _p(drop),
                                          _p(lits_b), B, int(t0), int(bool(add_bias)), _p(cs), _p(self.patch_w),
                                          _p(ws), self._stream()), "ytm_train_eval")
        return cs

    def train_update(self, cs: torch.Tensor, Y_b: torch.Tensor, lits_b: torch.Tensor, t0: int,
                     drop: torch.Tensor | None, sel_override: torch.Tensor | None = None,
                     counters: torch.Tensor | None = None) -> None:
        """Feedback of the batch.  counters: optional int64 [6] device tensor
        that accumulates the measurement counts of ytm_train_update_counted."""
        c = self._cfg_for(lits_b)
        B = lits_b.shape[0]
        ws = self.workspace(_lib.YTM_OP_TRAIN, B, c)
        with torch.cuda.device(self.device):
            if counters is None:
                check(self.lib.ytm_train_update(c, _p(self.state), _p(self.weights), _p(cs), _p(Y_b),
                                                _p(drop), _p(lits_b), B, int(t0), _p(sel_override), _p(self.patch_w),
                                                _p(ws), self._stream()),
                      "ytm_train_update")
            else:
                check(self.lib.ytm_train_update_counted(c, _p(self.state), _p(self.weights), _p(cs), _p(Y_b),
                                                        _p(drop), _p(lits_b), B, int(t0), _p(sel_override),
                                                        _p(self.patch_w), _p(ws), _p(counters), self._stream()),
                      "ytm_train_update_counted")

    def train_fit_b1(self, lits: torch.Tensor, Y: torch.Tensor, t0: int, drop: torch.Tensor | None) -> None:
        """Batch-1 training over all samples of lits in order (single
        process): one fused launch per sample."""
        c = self._cfg_for(lits)
        N = lits.shape[0]
        if N == 0:
            return
        ws = self.workspace(_lib.YTM_OP_TRAIN_B1, 0, c)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_train_fit_b1(c, _p(self.state), _p(self.weights), _p(self.bias), _p(drop),
                                            _p(lits), _p(Y), N, int(t0), _p(self.patch_w), _p(ws), self._stream()),
                  "ytm_train_fit_b1")

    def train_fit_batches(self, lits: torch.Tensor, Y: torch.Tensor, B: int, t0: int, drop: torch.Tensor | None,
                          add_bias: bool, comm=None, peer_ar=None) -> torch.Tensor:
        """Mini-batch training over all samples of lits in order, queued from C
        (eval, NCCL all-reduce of the class sums on `comm` if given, feedback
        per batch).  Returns the class sums [b, K] of the last batch."""
        c = self._cfg_for(lits)
        N = lits.shape[0]
        if N == 0:
            return torch.empty((0, self.K), dtype=torch.int32, device=self.device)
        B = int(min(B, N))
        ws = self.workspace(_lib.YTM_OP_TRAIN_LOOP, B, c)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_train_fit_batches(c, _p(self.state), _p(self.weights), _p(self.bias), _p(drop),
                                                 _p(lits), _p(Y), N, B, int(t0), int(bool(add_bias)),
                                                 _p(self.patch_w), comm, peer_ar, _p(ws), self._stream()),
                  "ytm_train_fit_batches")
        last = N - (N - 1) // B * B
        return ws[:last * self.K * 4].view(torch.int32).view(last, self.K)

    def b1_class_sums(self, N: int) -> torch.Tensor:
        """Class sums [1, K] the last train_fit_b1 call used for its last
        sample (slot (N-1) % 3 of the class-sum ring at the workspace start)."""
        ws = self._ws[_lib.YTM_OP_TRAIN_B1]
        ring = ws[:3 * self.K * 4].view(torch.int32).view(3, self.K)
        return ring[(N - 1) % 3].reshape(1, self.K)

    def selection(self, B: int) -> torch.Tensor:
        sel = torch.empty((B, self.C), dtype=torch.int32, device=self.device)
        ws = self.workspace(_lib.YTM_OP_TRAIN, B)
        with torch.cuda.device(self.device):
            check(self.lib.ytm_train_selection(self._cfg, B, _p(ws), _p(sel), self._stream()), "ytm_train_selection")
        return sel
