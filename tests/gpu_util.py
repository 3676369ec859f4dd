"""Helpers shared by the GPU tests: device buffers through torch (plumbing
only), and the per-row state struct of the operator ABI."""
import ctypes as C

import numpy as np
import torch

from mlxcat_b200 import _abi as A


def dev(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def ptr(t):
    return C.c_void_p(t.data_ptr())


class DeviceRows:
    """mlxcat_rows backed by torch tensors."""

    def __init__(self, histories, max_new, n_gen=None, active=None, temperature=None, top_p=None,
                 seed=None, has_seed=None, eos=None, trigger=None, hist_cap=None):
        R = len(histories)
        cap = hist_cap or (max(len(h) for h in histories) + 64)
        hist = np.zeros((R, cap), np.int32)
        for r, h in enumerate(histories):
            hist[r, :len(h)] = h
        self.hist = dev(hist)
        self.hist_len = dev(np.array([len(h) for h in histories], np.int32))
        self.kv_len = dev(np.array([max(len(h) - 1, 0) for h in histories], np.int32))
        self.n_gen = dev(np.array(n_gen if n_gen is not None else [1] * R, np.int32))
        self.max_new = dev(np.array(max_new, np.int32))
        self.active = dev(np.array(active if active is not None else [1] * R, np.int32))
        self.temperature = dev(np.array(temperature if temperature is not None else [0.0] * R, np.float32))
        self.top_p = dev(np.array(top_p if top_p is not None else [0.0] * R, np.float32))
        self.seed = dev(np.array(seed if seed is not None else [0] * R, np.uint64).view(np.int64))
        self.has_seed = dev(np.array(has_seed if has_seed is not None else [0] * R, np.int32))
        e = np.zeros((R, A.MAX_EOS), np.int32)
        ne = np.zeros(R, np.int32)
        for r in range(R):
            ids = (eos[r] if eos is not None else [])
            e[r, :len(ids)] = ids
            ne[r] = len(ids)
        self.eos = dev(e)
        self.n_eos = dev(ne)
        self.trigger = dev(np.array(trigger if trigger is not None else [-1] * R, np.int32))
        self.R = R
        self.cap = cap

    def struct(self):
        s = A.RowsC()
        s.hist = self.hist.data_ptr()
        s.hist_cap = self.cap
        s.rows = self.R
        for name in ("hist_len", "kv_len", "n_gen", "max_new", "active", "temperature", "top_p",
                     "seed", "has_seed", "eos", "n_eos", "trigger"):
            setattr(s, name, getattr(self, name).data_ptr())
        return s

    def history(self, r):
        n = int(self.hist_len[r].item())
        return self.hist[r, :n].cpu().numpy().tolist()
