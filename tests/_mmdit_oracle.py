"""The MMDiT model's numeric steps on the CPU oracle (oracle/eager.py) --
test infrastructure: ``imagine_b200.mmdit.MMDiT`` runs over this object in
the tests, and over ``NativeOps`` (libw8a8) in the product, so a difference
between the two is a difference between the kernels and the reference's
eager operators, not between two model codes.

Each step restates the reference's eager composition: ``adaln``
(inference/src/backend_eager.rs:176-236) then ``int8_linear``
(inference/src/int8_linear.rs:198-277); ``rms_rope``
(inference/src/backend_rope.rs:203-223) on the q / k heads; the residual
``addcmul`` (int8_linear.rs:99-112); attention as fp32 softmax(q k^T / sqrt d) v
rounded to bf16."""
from __future__ import annotations

import torch

from oracle import eager as O


class OracleOps:
    def quantize_weight(self, w):
        q, s = O.quantize_weight(w.cpu())
        return q.to(w.device), s.reshape(-1).to(w.device)

    def linear(self, x, p, act=None, residual=None, gate=None, input_norm=None, eps=1e-6):
        if input_norm is not None:
            return O.int8_linear(x, p.w, p.ws, p.b, torch.bfloat16, input_act="rms_norm",
                                 input_act_weight=input_norm, input_act_eps=eps, output_act=act)
        return O.int8_linear(x, p.w, p.ws, p.b, torch.bfloat16, residual=residual,
                             residual_scale=gate, output_act=act)

    def adaln_linear(self, x, scale, shift, p, act=None, eps=1e-6):
        return O.int8_linear(O.adaln(x, scale, shift, eps), p.w, p.ws, p.b, torch.bfloat16,
                             output_act=act)

    def adaln_qkv_rope(self, x, scale, shift, p, norm_w, freqs, rope_cols, eps=1e-6):
        y = O.int8_linear(O.adaln(x, scale, shift, eps), p.w, p.ws, p.b, torch.bfloat16)
        d = 128
        lead = y.shape[:-1]
        s = freqs.shape[0]
        heads = rope_cols // d
        qk = y[..., :rope_cols].reshape(-1, s, heads, d)
        w = norm_w.reshape(heads, d)
        # per-column norm weights: heads share one row per q / k half
        half = heads // 2
        q = qk[:, :, :half]
        k = qk[:, :, half:]
        qo, ko = O.rms_rope(q, k, freqs, w[0], w[half], eps)
        out = torch.cat([qo, ko], dim=2).reshape(*lead, rope_cols)
        return torch.cat([out, y[..., rope_cols:]], dim=-1)

    def row_absmax(self, x):
        return x.abs().amax(dim=-1).to(torch.float32).contiguous()

    def quantize_given_absmax(self, x, amax):
        q, s = O.quantize_int8_rowwise_given_absmax(x, amax.reshape(-1, 1))
        return q, s.reshape(-1)

    def gemm_s32(self, q, w):
        return O.int8_accumulate(q, w)

    def dequant(self, acc, xs, p, residual=None, gate=None, lead=None):
        y = O.dequant_eager(acc, xs, p.ws, p.b, torch.bfloat16)
        if lead is not None:
            y = y.reshape(*lead, -1)
        return O.apply_residual(y, residual, gate)

    def attention(self, joint, heads, head_dim):
        c = heads * head_dim
        return self.attention_split(joint[..., :c], joint[..., c:], heads, head_dim)

    def attention_split(self, q, kv, heads, head_dim):
        b = q.shape[0]
        c = heads * head_dim
        qh = q.float().unflatten(-1, (heads, head_dim)).transpose(1, 2)
        k, v = (kv[..., i * c:(i + 1) * c].float().unflatten(-1, (heads, head_dim)).transpose(1, 2)
                for i in range(2))
        a = torch.softmax(qh @ k.transpose(-1, -2) / head_dim ** 0.5, dim=-1)
        return (a @ v).transpose(1, 2).reshape(b, -1, c).to(torch.bfloat16)

    def adaln_qkv_rope_split(self, x, scale, shift, p, norm_w, freqs, q_outs, kv_outs, eps=1e-6):
        c = p.w.shape[0] // 3
        y = self.adaln_qkv_rope(x, scale, shift, p, norm_w, freqs, 2 * c, eps)
        for i in range(x.shape[0]):
            q_outs[i].copy_(y[i, :, :c])
            kv_outs[i].copy_(y[i, :, c:])

    def silu(self, x):
        return torch.nn.functional.silu(x)
