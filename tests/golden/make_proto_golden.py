"""Generate tests/golden/proto.npz from the LeanKV prototype (prototype/turboquant).

Run in a checkout that has the reference next to it:
    python tests/golden/make_proto_golden.py /path/to/LeanKV
The fixture holds, for seeded inputs: Lloyd-Max codebooks, rotation matrices,
TurboQuantizer.quantize / dequantize outputs for several configurations and the
tensors a multi-step LeanKVCache returns.  The GPU tests compare the CUDA path
against these numbers; nothing at test time imports the prototype.
"""
import os
import sys

import numpy as np
import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LEANKV_REF", "")
sys.path.insert(0, os.path.join(REF, "prototype"))
from turboquant import lloyd_max, rotation  # noqa: E402
from turboquant.kv_cache import LeanKVCache  # noqa: E402
from turboquant.quantizer import TurboQuantizer  # noqa: E402

out = {}
for bits in (2, 3, 4):
    for dim in (64, 128, 256):
        lv, bd = lloyd_max.get_precomputed_codebook(bits, dim)
        out[f"cb_{bits}_{dim}_levels"] = lv.numpy()
        out[f"cb_{bits}_{dim}_bounds"] = bd.numpy()
out["rot_hadamard_64"] = rotation.hadamard_matrix(64).numpy()
out["rot_randhad_128_s43_row0"] = rotation.randomized_hadamard(128, seed=43)[0].numpy()
out["rot_orth_64_s7"] = rotation.random_orthogonal(64, seed=7).numpy()

CASES = [  # name, head_dim, bits, group_size, strategy, qjl, layer
    ("a", 128, 3, None, "randomized_hadamard", True, 1),
    ("b", 64, 4, 16, "hadamard", False, 0),
    ("c", 64, 2, None, "random_orthogonal", True, 0),
    ("d", 256, 3, 32, "randomized_hadamard", True, 1),
    ("e", 32, 4, None, "randomized_hadamard", False, 0),
]
for name, hd, bits, gs, strat, qjl, layer in CASES:
    torch.manual_seed(100 + hd)
    x = torch.randn(1, 2, 16, hd)
    x[..., :2] *= 8.0
    tq = TurboQuantizer(n_layers=2, head_dim=hd, bits=bits, group_size=gs, rotation_strategy=strat,
                        use_qjl=qjl, seed=42)
    q = tq.quantize(x, layer)
    out[f"q{name}_x"] = x.numpy()
    out[f"q{name}_idx"] = q.indices.numpy()
    out[f"q{name}_norms"] = q.norms.numpy()
    if qjl:
        out[f"q{name}_signs"] = q.qjl_signs.numpy()
        out[f"q{name}_mean"] = q.qjl_mean_abs.numpy()
    out[f"q{name}_deq"] = tq.dequantize(q, layer).numpy()
    out[f"q{name}_deq_inv"] = tq.dequantize(q, layer, apply_inverse_rot=True).numpy()
    if strat == "random_orthogonal":
        out[f"q{name}_rot"] = tq.rotations[layer].numpy()
    out[f"q{name}_qrot"] = tq.quantize_for_attention(x[:, :, :3], layer).numpy()

for vrot in ("none", "randomized_hadamard"):
    torch.manual_seed(5)
    cache = LeanKVCache(n_layers=2, head_dim=64, n_kv_heads=2, k_bits=3, v_bits=4, v_rotation=vrot)
    steps = [5, 1, 1]
    ks, vs = [], []
    for n in steps:
        for layer in range(2):
            k = torch.randn(2, 2, n, 64)
            v = torch.randn(2, 2, n, 64)
            ks.append(k)
            vs.append(v)
            ak, av = cache.update(k, v, layer)
    tag = "kvn" if vrot == "none" else "kvr"
    out[f"{tag}_k_in"] = torch.stack([torch.cat(ks[l::2], 2) for l in range(2)]).numpy()
    out[f"{tag}_v_in"] = torch.stack([torch.cat(vs[l::2], 2) for l in range(2)]).numpy()
    out[f"{tag}_keys_l1"] = ak.numpy()
    out[f"{tag}_values_l1"] = av.numpy()
    out[f"{tag}_len"] = np.array(cache.get_seq_length())

dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "proto.npz")
np.savez_compressed(dst, **out)
print("wrote", dst, len(out), "arrays", os.path.getsize(dst), "bytes")
