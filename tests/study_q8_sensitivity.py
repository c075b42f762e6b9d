"""Sensitivity of futon's Q8 path to float32-level perturbations (a study,
not a test; run by hand: python tests/study_q8_sensitivity.py, ~3 min CPU).

Runs the arctic-shaped encoder's Q8 forward (quant.go scheme, float64
emulation via torch_ref) on two sequences, once exactly and then with
(a) split-bf16 attention (hi+lo operands, the precision of the library's
int8-path attention kernel) and (b) multiplicative noise of relative size
1e-7 … 1e-4 injected into every attention output. Measured:
    split      cos ≈ 0.99986-0.99987
    noise 1e-7 cos ≈ 0.99990-0.99991
    noise 1e-6 cos ≈ 0.99986
i.e. any implementation that is not bit-identical to the reference's Q8
path lands near 1 − cos ≈ 1.4e-4 from it: int8 rounding boundaries amplify
rounding-level differences through 48 quantisations. The float path under
the same perturbations stays at cos ≥ 0.9999999.
"""
import math
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
sys.path.insert(0, str(Path(__file__).resolve().parent))
from futon_b200 import synth
import torch_ref as TR
cfg=synth.arch('arctic'); w=synth.make_weights(cfg)
rng=np.random.default_rng(5)
seqs=[np.concatenate([[101],rng.integers(1000,cfg.vocab_size,L-2),[102]]) for L in (256,200)]
def bf(x): return x.to(torch.bfloat16).to(x.dtype)
def split(x): hi=bf(x.float()).double(); lo=bf((x-hi).float()).double(); return hi,lo
def smm(eq,a,b):
    ah,al=split(a); bh,bl=split(b)
    return torch.einsum(eq,ah,bh)+torch.einsum(eq,ah,bl)+torch.einsum(eq,al,bh)
class Emu(TR.TorchRef):
    mode='exact'; noise=0.0
    @torch.no_grad()
    def encode(self, ids, out_dim=0):
        cfg,t=self.cfg,self.t; h,H,hd=cfg.hidden_size,cfg.num_heads,self.hd
        ids_t=torch.as_tensor(np.asarray(ids,dtype=np.int64)); L=ids_t.numel()
        x=t["embeddings.word"][ids_t]+t["embeddings.token_type"][0]
        x=self._ln(x,t["embeddings.norm.weight"],t["embeddings.norm.bias"],cfg.layer_norm_eps)
        g=torch.Generator().manual_seed(0)
        for li in range(cfg.num_layers):
            p=f"layers.{li}."
            qkv=self._mm(x,p+"attn.qkv.weight",None).float().double()
            q=qkv[:,:h].reshape(L,H,hd); k=qkv[:,h:2*h].reshape(L,H,hd); v=qkv[:,2*h:].reshape(L,H,hd)
            q,k=self._rot(q,L),self._rot(k,L)
            if self.mode=='split':
                s=smm("qhd,khd->hqk",q,k)/math.sqrt(hd)
                pr=torch.softmax(s,dim=-1)
                o=smm("hqk,khd->qhd",pr,v).reshape(L,h)
            else:
                s=torch.einsum("qhd,khd->hqk",q,k)/math.sqrt(hd); pr=torch.softmax(s,dim=-1)
                o=torch.einsum("hqk,khd->qhd",pr,v).reshape(L,h)
                if self.noise: o=o*(1+self.noise*torch.randn(o.shape,generator=g,dtype=o.dtype))
            o=o.float().double()
            a=self._mm(o,p+"attn.out.weight",None)+x
            x=self._ln(a,t[p+"norm1.weight"],t[p+"norm1.bias"],cfg.layer_norm_eps)
            f=self._mm(x,p+"mlp.fc1.weight",None); gg=self._mm(x,p+"mlp.gate.weight",None)
            f=f*(gg*torch.sigmoid(gg))
            y=self._mm(f,p+"mlp.fc2.weight",None)+x
            x=self._ln(y,t[p+"norm2.weight"],t[p+"norm2.bias"],cfg.layer_norm_eps)
        pooled=x[0]; return (pooled/pooled.norm()).numpy()
def run(mode='exact',noise=0.0):
    m=Emu(cfg,w,dtype=torch.float64,q8=True); m.mode=mode; m.noise=noise
    return np.stack([m.encode(s) for s in seqs])
cos=lambda a,b:((a*b).sum(1)/np.linalg.norm(a,axis=1)/np.linalg.norm(b,axis=1))
A=run()
print('split', cos(A,run('split')), flush=True)
for n in (1e-7,1e-6,1e-5,1e-4): print('noise',n, cos(A,run(noise=n)), flush=True)
