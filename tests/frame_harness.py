"""Shared set-up for the frame parity tests: device buffers (torch on cuda:0) holding
the same seeded inputs the CPU oracle gets, and zero-copy views of device pointers."""
from __future__ import annotations

import numpy as np
import torch

from navi_b200 import engine
from oracle import model as om


class DevView:
    """Zero-copy torch view of a device pointer (float32 or uint16)."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def dev_f32(ptr: int, n: int) -> np.ndarray:
    return torch.as_tensor(DevView(ptr, n), device="cuda").cpu().numpy().copy()


def oracle_sampling(s: engine.Sampling) -> om.Sampling:
    return om.Sampling(s.temperature, s.top_k, s.top_p, s.repetition_penalty, s.cp_temperature, s.cp_top_k, s.cp_top_p,
                       s.min_frames, s.rng)


class Setup:
    """A device, uploaded weights, a frame, and a seeded KV cache mirrored for the oracle."""

    def __init__(self, navi_path: str, max_pos: int = 256, deadline_us: int = 0):
        self.dev = engine.Device(0)
        self.w = engine.Weights(self.dev, navi_path)
        self.frame = engine.Frame(self.dev, self.w, deadline_us=deadline_us)
        self.W = om.Weights.from_navi(navi_path)
        p = self.w.params
        self.H, self.TV, self.CV = p.talker.hidden, p.talker.vocab, p.cp.vocab
        self.kv_dim = p.talker.n_kv_head * p.talker.head_dim
        self.n_layer = p.talker.n_layer
        self.max_pos = max_pos
        self.k = [torch.zeros(max_pos, self.kv_dim, dtype=torch.float16, device="cuda") for _ in range(self.n_layer)]
        self.v = [torch.zeros(max_pos, self.kv_dim, dtype=torch.float16, device="cuda") for _ in range(self.n_layer)]
        self.kv = engine.KvCache.wrap([t.data_ptr() for t in self.k], [t.data_ptr() for t in self.v], max_pos, self.kv_dim,
                                      keepalive=(self.k, self.v))

    def fill_kv(self, n: int, seed: int) -> None:
        g = torch.Generator().manual_seed(seed)
        for l in range(self.n_layer):
            self.k[l][:n] = torch.randn(n, self.kv_dim, generator=g).half().cuda()
            self.v[l][:n] = torch.randn(n, self.kv_dim, generator=g).half().cuda()

    def oracle_kv(self):
        return [(self.k[l].float().cpu().clone(), self.v[l].float().cpu().clone()) for l in range(self.n_layer)]

    def step_out(self) -> np.ndarray:
        return dev_f32(self.frame.d_step_out(), self.H)
