"""Generate the golden fixtures of tests/golden/ from the reference's PyTorch path.

    python tests/golden/make_golden.py

The reference's own golden generator (tests/engine_ref.py) needs the real Qwen3.5-0.8B checkpoint and tokenizer,
which are not available offline; its method is kept: run Hugging Face transformers (5.5.0 here) in fp32 on the CPU
with the same hooks (a down_proj forward-pre hook for neuron pushes, a layer forward hook for the residual vector),
on seeded inputs, and store the outputs.  The fla / causal-conv1d fast paths are forced off so the pure-torch
reference functions run.  Fixtures:

  gdn_ops.npz     torch_chunk_gated_delta_rule / torch_recurrent_gated_delta_rule / torch_causal_conv1d_update on
                  seeded inputs (ragged T = 100, an initial state, in-kernel l2norm)
  tiny_model.npz  a tiny Qwen3.5 model (tests/golden/tiny.py weights) run through Qwen3_5ForCausalLM: prefill of
                  3 rows with per-row pushes and vectors, then 6 greedy steps (logits and tokens)
  rope.npz        the text rotary table (cos / sin) of Qwen3_5TextRotaryEmbedding at a few positions
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from oracle import hf  # noqa: E402
from oracle.model import Cfg  # noqa: E402
from tiny import TINY, tiny_state_dict, tiny_workload  # noqa: E402


def gdn_ops():
    M = hf._modeling()
    g = torch.Generator().manual_seed(11)
    B, T, H, d = 2, 100, 2, 128
    q = torch.randn(B, T, H, d, generator=g)
    k = torch.randn(B, T, H, d, generator=g)
    v = torch.randn(B, T, H, d, generator=g)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    gg = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=g))
    s0 = torch.randn(B, H, d, d, generator=g) * 0.05
    oc, sc = M.torch_chunk_gated_delta_rule(q, k, v, gg, beta, initial_state=s0.clone(), output_final_state=True,
                                            use_qk_l2norm_in_kernel=True)
    orr, sr = M.torch_recurrent_gated_delta_rule(q, k, v, gg, beta, initial_state=s0.clone(), output_final_state=True,
                                                 use_qk_l2norm_in_kernel=True)
    C, KS, Tc = 256, 4, 5
    xc = torch.randn(B, C, Tc, generator=g)
    wc = torch.randn(C, KS, generator=g) * 0.3
    state = torch.randn(B, C, KS, generator=g)  # HF keeps KS inputs; the first is never used
    state_in = state.clone()
    outc = M.torch_causal_conv1d_update(xc.clone(), state, wc, None, "silu")
    np.savez_compressed(os.path.join(HERE, "gdn_ops.npz"), q=q.numpy(), k=k.numpy(), v=v.numpy(), beta=beta.numpy(),
                        g=gg.numpy(), s0=s0.numpy(), o_chunk=oc.numpy(), s_chunk=sc.numpy(), o_rec=orr.numpy(),
                        s_rec=sr.numpy(), conv_x=xc.numpy(), conv_w=wc.numpy(), conv_state_in=state_in.numpy(),
                        conv_out=outc.numpy(), conv_state_out=state.numpy())


def tiny_model():
    sd_np, types = tiny_state_dict()
    c = TINY
    cfg = Cfg(hidden=c["hidden"], inter=c["inter"], vocab=c["vocab"], layers=c["layers"], nh=c["nh"], nkv=c["nkv"],
              hd=c["hd"], rot=c["rot"], theta=c["theta"], hk=c["hk"], hv=c["hv"], dk=c["dk"], dv=c["dv"], ks=c["ks"],
              eps=c["eps"], layer_types=types)
    model = hf.build_model(cfg, seed=0)
    sd = {k: torch.from_numpy(v) for k, v in sd_np.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("lm_head" in m for m in missing), (missing, unexpected)
    hooks = hf.Hooks(model)
    ids, push, vec_layer, vecs = tiny_workload()
    hpush = {l: [(r["n"], r["mode"], torch.tensor(r["vals"])) for r in recs] for l, recs in push.items()}
    first, steps, toks = hf.prefill_and_greedy(model, torch.from_numpy(ids), 6, hooks, push=hpush,
                                               vec=(vec_layer, torch.from_numpy(vecs)))
    plain_first, plain_steps, plain_toks = hf.prefill_and_greedy(model, torch.from_numpy(ids), 6, hooks)
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), ids=ids, logits_prefill=first.numpy(),
                        logits_steps=torch.stack(steps).numpy(), tokens=toks.numpy(),
                        plain_logits_prefill=plain_first.numpy(), plain_logits_steps=torch.stack(plain_steps).numpy(),
                        plain_tokens=plain_toks.numpy(),
                        versions=np.array([torch.__version__, __import__("transformers").__version__]))


def rope():
    M = hf._modeling()
    cfg = hf.hf_config(Cfg())
    emb = M.Qwen3_5TextRotaryEmbedding(cfg)
    pos = torch.tensor([[0, 1, 2, 63, 64, 1000, 4095, 16383]])
    cos, sin = emb(torch.zeros(1, dtype=torch.float32), pos)
    np.savez_compressed(os.path.join(HERE, "rope.npz"), pos=pos.numpy(), cos=cos.numpy(), sin=sin.numpy())


if __name__ == "__main__":
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    gdn_ops()
    tiny_model()
    rope()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
