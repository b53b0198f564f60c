"""CPU test double of qik.parallel.QikOps built on the oracle (test infrastructure).

Lets the parallel layer's sharding, collectives and algebra run as gloo ranks on
CPU: the same method contract as the CUDA ops, computed by the CPU restatement."""
import numpy as np
import torch

from oracle import oracle as O


def _bits_to_float(t: torch.Tensor) -> float:
    return float(np.array([int(t.reshape(-1)[0].item())], dtype=np.int32).view(np.float32)[0])


def _float_to_bits(v: float) -> int:
    return int(np.array([v], dtype=np.float32).view(np.int32)[0])


class OracleOps:
    def amax_bits(self, x):
        return torch.tensor([_float_to_bits(O.amax(x.contiguous()))], dtype=torch.int32)

    def zeros_amax(self, device):
        return torch.zeros(1, dtype=torch.int32)

    def pack(self, x, amax):
        s = O.scale_from_amax(_bits_to_float(amax), O.SCALE_CUDA)
        bits = x.contiguous().view(torch.int16).numpy().view(np.uint16)
        q = np.empty(bits.shape, dtype=np.uint8)
        O.lib().qik_oracle_pack_act_bf16(bits.ctypes.data, bits.size, O.act_reciprocal(s), q.ctypes.data)
        return torch.from_numpy(q).view(torch.float8_e4m3fn), torch.tensor([s], dtype=torch.float32)

    def gemm(self, xq, sx, wq, sw, bias=None, out_dtype=torch.bfloat16, epilogue=0, amax_out=None):
        y = O.fp8_linear(xq, float(sx.reshape(-1)[0]), wq, float(sw.reshape(-1)[0]), bias)
        if out_dtype == torch.float32:
            return y
        y = y.to(torch.bfloat16)
        if epilogue == 1:
            y = O.gelu_tanh(y)
        if amax_out is not None:
            cur = _bits_to_float(amax_out)
            amax_out.fill_(_float_to_bits(max(cur, y.float().abs().max().item())))
        return y

    def attention(self, q, k, v, L):
        return O.block_causal_attention(q, k, v, L)

    def bias_bf16(self, x, bias, amax):
        y = x.float() + (bias.float() if bias is not None else 0.0)
        y = y.to(torch.bfloat16)
        cur = _bits_to_float(amax)
        amax.fill_(_float_to_bits(max(cur, y.float().abs().max().item())))
        return y
