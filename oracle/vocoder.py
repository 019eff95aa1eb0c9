"""CPU oracle of the vocoder (codec decoder) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this
module, and only as the checker (or the timed CPU baseline); the product path never
does.

A plain PyTorch fp32 (CPU) restatement of the reference's streaming codec decoder,
model/qwen3tts/vocoder.hip, on f16-rounded weights upcast to f32:

  decode_chunk       vocoder.hip:261-343: rvq -> rvq output projections -> pre_conv
                     (k=3) -> input_proj -> pre-transformer layers -> norm ->
                     output_proj -> 2 x (transposed conv k=s + ConvNeXt) -> dec0 (k=7)
                     -> 4 x (SnakeBeta, transposed conv k=2s, 3 residual units
                     dil 1/3/9) -> SnakeBeta -> final conv (k=7) -> clamp [-1, 1]
  rvq                vocoder.hip:113-131 (first codebook row | sum of the 15 rest rows)
  causal conv        kernels.h:72-242 (y[t] = b + sum_j W[:, :, j] x[t - (K-1-j) dil],
                     rows before the chunk come from the conv's own input history)
  transposed conv    vocoder.hip:373-385 (out[i s + p] = b + sum_m W[:, :, p + m s] x[i - m])
  pre-transformer    vocoder.hip:275-291, 59-111 (RMSNorm, no q/k norm, rotate-half
                     RoPE, sliding-window causal attention over keys (pos - window, pos],
                     layer scales on the attention and MLP residual branches)
  ConvNeXt           vocoder.hip:20-56, 310-326 (depthwise k=7 + LayerNorm eps 1e-6,
                     pwconv1 + erf GELU, pwconv2, gamma, residual)
  SnakeBeta          x + sin(x e^alpha)^2 / (e^beta + 1e-9) (vocoder.hip:453-461)
  history            vocoder.hip:133-141, 245-251: each conv keeps the last (K-1) dil
                     rows of its raw input; reset() zeroes them (vocoder.hip:618-629)

The reference's own vocoder test pins it against qwen-tts with the released
checkpoint (tests/reference/vocoder16_pcm.npy), which needs weights that are not
available here: parity unpinned at that boundary.  tests/ pin the pieces of this
module against independent torch formulations instead (conv_transpose1d, padded
conv1d, dense masked attention) and check chunked decoding against one-shot.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from oracle.model import rmsnorm, rope_inv_freq, silu

DEC = "codec.decoder."


def snake_coeffs(alpha: torch.Tensor, beta: torch.Tensor):
    """(e^alpha, 1 / (e^beta + 1e-9)) in f32 (vocoder.hip:453-461)."""
    return torch.exp(alpha.float()), 1.0 / (torch.exp(beta.float()) + 1e-9)


def snake(x: torch.Tensor, ea: torch.Tensor, ib: torch.Tensor) -> torch.Tensor:
    s = torch.sin(x * ea)
    return x + s * s * ib


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))


class Vocoder:
    """Streaming decoder state: per-conv input histories, the pre-transformer's K/V
    rows and the position counter. decode() appends samples_per_frame * T samples."""

    def __init__(self, W, window: int | None = None) -> None:
        self.W = W
        c = W.cfg
        self.c = c
        v = c.vocoder
        self.VH, self.nh, self.hd, self.ff, self.eps, self.theta = v.hidden, v.n_head, v.head_dim, v.ff, v.eps, v.rope_theta
        self.n_layer = v.n_layer
        self.window = c.sliding_window if window is None else window
        self.reset()

    def reset(self) -> None:
        self.pos0 = 0
        self.hist = {}
        HD = self.nh * self.hd
        self.kc = [torch.zeros(0, HD) for _ in range(self.n_layer)]
        self.vc = [torch.zeros(0, HD) for _ in range(self.n_layer)]

    # --- convolutions with carried input history -------------------------------------------

    def _with_hist(self, name: str, x: torch.Tensor, H: int) -> torch.Tensor:
        """[H rows of history; x]; the history becomes the last H rows of that."""
        if H == 0:
            return x
        h = self.hist.get(name)
        if h is None:
            h = torch.zeros(H, x.shape[1])
        full = torch.cat([h, x], 0)
        self.hist[name] = full[-H:].clone()
        return full

    def conv(self, name: str, x: torch.Tensor, w: torch.Tensor, b, dil: int = 1, pro=None) -> torch.Tensor:
        """Causal Conv1d of x[T, Cin] with w[Cout, Cin, K] (kernels.h:72-242)."""
        K = w.shape[2]
        full = self._with_hist(name, x, (K - 1) * dil)
        if pro is not None:
            full = pro(full)
        return F.conv1d(full.T.unsqueeze(0), w, b, dilation=dil)[0].T

    def trans_conv(self, name: str, x: torch.Tensor, w: torch.Tensor, b, s: int, pro=None) -> torch.Tensor:
        """Causal transposed conv, stride s, w[Cin, Cout, k] with k a multiple of s:
        out[i s + p] = b + sum_m x[i - m] W[:, :, p + m s] (vocoder.hip:373-385)."""
        kk = w.shape[2] // s
        H = kk - 1
        full = self._with_hist(name, x, H)
        if pro is not None:
            full = pro(full)
        T, Cout = x.shape[0], w.shape[1]
        out = torch.empty(T, s, Cout)
        for p in range(s):
            acc = b.expand(T, Cout).clone() if b is not None else torch.zeros(T, Cout)
            for m in range(kk):
                acc = acc + full[H - m:H - m + T] @ w[:, :, p + m * s]
            out[:, p] = acc
        return out.reshape(T * s, Cout)

    # --- stages -------------------------------------------------------------------------------

    def rvq(self, codes: torch.Tensor) -> torch.Tensor:
        """codes[T, n_q] -> rvq output [T, codebook_dim] (vocoder.hip:113-131, 264-265)."""
        W, c = self.W, self.c
        q = DEC + "quantizer."
        first = W[q + "rvq_first.vq.layers.0._codebook.codebook"][codes[:, 0]]
        rest = torch.zeros_like(first)
        for i in range(1, c.vq_n_q):
            rest = rest + W[f"{q}rvq_rest.vq.layers.{i - 1}._codebook.codebook"][codes[:, i]]
        return first @ W[q + "rvq_first.output_proj.weight"][:, :, 0].T + rest @ W[q + "rvq_rest.output_proj.weight"][:, :, 0].T

    def attention_layer(self, l: int, x: torch.Tensor) -> torch.Tensor:
        W = self.W
        p = f"{DEC}pre_transformer.layers.{l}."
        T = x.shape[0]
        nh, hd = self.nh, self.hd
        inv = rope_inv_freq(hd, self.theta)
        n = rmsnorm(x, W[p + "input_layernorm.weight"], self.eps)
        q = (n @ W[p + "self_attn.q_proj.weight"].T).view(T, nh, hd)
        k = (n @ W[p + "self_attn.k_proj.weight"].T).view(T, nh, hd)
        v = (n @ W[p + "self_attn.v_proj.weight"].T).view(T, nh, hd)
        pos = torch.arange(self.pos0, self.pos0 + T, dtype=torch.float32)
        ang = pos[:, None] * inv[None, :]                     # f32 product, as k_rope_append
        cs, sn = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
        half = hd // 2

        def rot(z):
            z0, z1 = z[..., :half], z[..., half:]
            return torch.cat([z0 * cs - z1 * sn, z1 * cs + z0 * sn], -1)
        q, k = rot(q), rot(k)
        self.kc[l] = torch.cat([self.kc[l], k.reshape(T, -1)], 0)
        self.vc[l] = torch.cat([self.vc[l], v.reshape(T, -1)], 0)
        K = self.kc[l].view(-1, nh, hd)
        V = self.vc[l].view(-1, nh, hd)
        scale = 1.0 / math.sqrt(hd)
        att = torch.empty(T, nh, hd)
        for t in range(T):
            ps = self.pos0 + t
            k0 = max(0, ps - self.window + 1)
            for h in range(nh):
                s = (K[k0:ps + 1, h] @ q[t, h]) * scale
                att[t, h] = torch.softmax(s, 0) @ V[k0:ps + 1, h]
        x = x + (att.reshape(T, -1) @ W[p + "self_attn.o_proj.weight"].T) * W[p + "self_attn_layer_scale.scale"]
        n2 = rmsnorm(x, W[p + "post_attention_layernorm.weight"], self.eps)
        a = silu(n2 @ W[p + "mlp.gate_proj.weight"].T) * (n2 @ W[p + "mlp.up_proj.weight"].T)
        return x + (a @ W[p + "mlp.down_proj.weight"].T) * W[p + "mlp_layer_scale.scale"]

    def convnext(self, j: int, x: torch.Tensor) -> torch.Tensor:
        """Depthwise k=7 conv + LayerNorm + pwconv1 (GELU) + pwconv2 * gamma + residual."""
        W = self.W
        up = f"{DEC}upsample.{j}.1."
        full = self._with_hist(f"cnx{j}", x, 6)
        y = F.conv1d(full.T.unsqueeze(0), W[up + "dwconv.conv.weight"], W[up + "dwconv.conv.bias"], groups=x.shape[1])[0].T
        mu = y.mean(-1, keepdim=True)
        var = ((y - mu) ** 2).mean(-1, keepdim=True)
        y = (y - mu) * torch.rsqrt(var + 1e-6) * W[up + "norm.weight"] + W[up + "norm.bias"]
        g = gelu_erf(y @ W[up + "pwconv1.weight"].T + W[up + "pwconv1.bias"])
        return (g @ W[up + "pwconv2.weight"].T + W[up + "pwconv2.bias"]) * W[up + "gamma"] + x

    def decode_chunk(self, codes, stages: dict | None = None) -> torch.Tensor:
        """codes[T, n_q] (ints) -> pcm [T * samples_per_frame] f32 (vocoder.hip:261-343).
        stages, when given, receives the intermediate activations by name."""
        W, c = self.W, self.c
        codes = torch.as_tensor(codes, dtype=torch.long).reshape(-1, c.vq_n_q)
        T = codes.shape[0]
        keep = (lambda k, v: stages.__setitem__(k, v.clone())) if stages is not None else (lambda k, v: None)
        h = self.rvq(codes)
        keep("rvq", h)
        a = self.conv("pre_conv", h, W[DEC + "pre_conv.conv.weight"], W[DEC + "pre_conv.conv.bias"])
        keep("pre_conv", a)
        pt = DEC + "pre_transformer."
        x = a @ W[pt + "input_proj.weight"].T + W[pt + "input_proj.bias"]
        for l in range(self.n_layer):
            x = self.attention_layer(l, x)
            keep(f"layer{l}", x)
        x = rmsnorm(x, W[pt + "norm.weight"], self.eps)
        u = x @ W[pt + "output_proj.weight"].T + W[pt + "output_proj.bias"]
        keep("pre_transformer", u)
        for j, r in enumerate(c.upsampling_ratios):
            up = f"{DEC}upsample.{j}."
            u = self.trans_conv(f"up{j}", u, W[up + "0.conv.weight"], W[up + "0.conv.bias"], r)
            u = self.convnext(j, u)
            keep(f"up{j}", u)
        d = self.conv("dec0", u, W[DEC + "decoder.0.conv.weight"], W[DEC + "decoder.0.conv.bias"])
        keep("dec0", d)
        for b, rate in enumerate(c.upsample_rates):
            bp = f"{DEC}decoder.{b + 1}.block."
            ea, ib = snake_coeffs(W[bp + "0.alpha"], W[bp + "0.beta"])
            P = self.trans_conv(f"blk{b}.up", d, W[bp + "1.conv.weight"], W[bp + "1.conv.bias"], rate,
                                pro=lambda z, ea=ea, ib=ib: snake(z, ea, ib))
            for k, dil in enumerate((1, 3, 9)):
                rp = f"{bp}{2 + k}."
                a1, b1 = snake_coeffs(W[rp + "act1.alpha"], W[rp + "act1.beta"])
                a2, b2 = snake_coeffs(W[rp + "act2.alpha"], W[rp + "act2.beta"])
                Q = self.conv(f"blk{b}.u{k}.c1", P, W[rp + "conv1.conv.weight"], W[rp + "conv1.conv.bias"], dil,
                              pro=lambda z, a1=a1, b1=b1: snake(z, a1, b1))
                P = P + self.conv(f"blk{b}.u{k}.c2", Q, W[rp + "conv2.conv.weight"], W[rp + "conv2.conv.bias"], 1,
                                  pro=lambda z, a2=a2, b2=b2: snake(z, a2, b2))
            keep(f"dec{b + 1}", P)
            d = P
        n = len(c.upsample_rates)
        ea, ib = snake_coeffs(W[f"{DEC}decoder.{n + 1}.alpha"], W[f"{DEC}decoder.{n + 1}.beta"])
        y = self.conv("final", d, W[f"{DEC}decoder.{n + 2}.conv.weight"], W[f"{DEC}decoder.{n + 2}.conv.bias"], 1,
                      pro=lambda z: snake(z, ea, ib))
        self.pos0 += T
        return y.clamp(-1.0, 1.0).reshape(-1)

    def decode(self, codes, n_frames: int, max_chunk: int) -> torch.Tensor:
        """Vocoder::decode (vocoder.hip:632-651): chunks of at most max_chunk frames."""
        codes = torch.as_tensor(codes, dtype=torch.long).reshape(-1, self.c.vq_n_q)[:n_frames]
        outs = [self.decode_chunk(codes[f0:f0 + max_chunk]) for f0 in range(0, n_frames, max_chunk)]
        return torch.cat(outs) if outs else torch.zeros(0)
