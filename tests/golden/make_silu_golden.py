"""Golden SiLU tables for the fused SiLU-and-mul quantizer: the silu that
vLLM's ``silu_and_mul`` (``torch.ops._C.silu_and_mul``, vllm 0.22) produces
for every bf16 and every f16 gate bit pattern, with the up half set to 1.

Needs a CUDA device.  Falls back to torch's ``F.silu`` in fp32 rounded to
the dtype when vLLM's compiled ops are missing; on a B200 the two agree on
all 2 x 65536 patterns (``torch_equals_vllm`` records it).

    python tests/golden/make_silu_golden.py     # writes tests/golden/silu_golden.npz
"""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def silu_table(dtype, use_vllm):
    n = 65536
    gate = torch.arange(n, dtype=torch.int32).to(torch.int16).view(dtype).cuda()
    torch_silu = torch.nn.functional.silu(gate.float()).to(dtype)
    if not use_vllm:
        return torch_silu.view(torch.int16).cpu().numpy().view(np.uint16), None
    x = torch.cat([gate.view(1, n), torch.ones(1, n, dtype=dtype, device="cuda")], dim=1)
    out = torch.empty(1, n, dtype=dtype, device="cuda")
    torch.ops._C.silu_and_mul(out, x)
    a, b = out.view(-1), torch_silu
    same = (a.view(torch.int16) == b.view(torch.int16)) | (torch.isnan(a.float()) & torch.isnan(b.float()))
    return out.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), bool(same.all())


def main():
    try:
        import vllm._custom_ops  # noqa: F401  registers torch.ops._C
        use_vllm = hasattr(torch.ops._C, "silu_and_mul")
    except Exception:
        use_vllm = False
    bf16, eq_b = silu_table(torch.bfloat16, use_vllm)
    f16, eq_h = silu_table(torch.float16, use_vllm)
    np.savez_compressed(os.path.join(HERE, "silu_golden.npz"), bf16=bf16, f16=f16,
                        source=np.array("vllm silu_and_mul" if use_vllm else "torch F.silu"),
                        torch_equals_vllm=np.array([eq_b, eq_h]))
    print("source", "vllm" if use_vllm else "torch", "torch==vllm", eq_b, eq_h)


if __name__ == "__main__":
    main()
