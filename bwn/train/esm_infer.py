"""ESM-2 masked-residue inference (``contrib/esm2/run_esm.py:72-186``): mask
the middle residue of each sequence, run the model (tensor-parallel across
the ranks when launched with several), report the predicted residue.

    python -m bwn.train.esm_infer --size 650M
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m bwn.train.esm_infer --size 15B
"""
from __future__ import annotations

import argparse
import json

import torch

from ..config import ESM2_SIZES, ESM_ALPHABET, ESM2Config

DEFAULT_SEQUENCES = [
    "MKTVRQERLKSIVRILERSKEPVSGAQLAEELSVSRQVIVQDIAYLRSLGYNIVATPRGYVLAGG",
    "KALTARQQEVFDLIRDHISQTGMPPTRAEIAQRLGFRSPNAAEEHLKALARKGVIEIVSGASRGIRLLQEE",
]


def tokenize(seqs: list[str], cfg: ESM2Config, max_len: int | None = None):
    """ESM alphabet ids with ``<cls>``/``<eos>``, right-padded with ``<pad>``;
    ``<mask>`` in a sequence string is one token, letters outside the alphabet
    are ``<unk>`` (as the HF ESM tokenizer maps them)."""
    idx = {t: i for i, t in enumerate(ESM_ALPHABET)}
    rows = []
    for s in seqs:
        toks, i = [cfg.cls_token_id], 0
        while i < len(s):
            if s.startswith("<mask>", i):
                toks.append(cfg.mask_token_id)
                i += 6
            else:
                toks.append(idx.get(s[i], idx["<unk>"]))
                i += 1
        toks.append(cfg.eos_token_id)
        rows.append(toks)
    L = max_len or max(len(r) for r in rows)
    ids = torch.full((len(rows), L), cfg.pad_token_id, dtype=torch.long)
    am = torch.zeros(len(rows), L, dtype=torch.long)
    for b, r in enumerate(rows):
        r = r[:L]
        ids[b, :len(r)] = torch.tensor(r)
        am[b, :len(r)] = 1
    return ids, am


@torch.no_grad()
def predict_masked_middle(model, seqs: list[str], max_len: int | None = None) -> list[dict]:
    cfg = model.cfg
    dev = next(model.parameters()).device
    masked, mids = [], []
    for s in seqs:
        m = len(s) // 2
        masked.append(s[:m] + "<mask>" + s[m + 1:])
        mids.append(m)
    ids, am = tokenize(masked, cfg, max_len)
    logits = model(ids.to(dev), am.to(dev)).float()
    out = []
    for b, (s, m) in enumerate(zip(seqs, mids)):
        p = torch.softmax(logits[b, m + 1], -1)  # +1: <cls>
        top = int(p.argmax())
        out.append({"position": m, "true": s[m], "predicted": ESM_ALPHABET[top], "prob": float(p[top])})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", "--model-size", default="8M", choices=sorted(ESM2_SIZES))
    ap.add_argument("--checkpoint", default="", help="HF safetensors directory (random init when empty)")
    ap.add_argument("--max-len", "--max-seq-len", type=int, default=128, help="padded length")
    ap.add_argument("--sequences", nargs="+", default=None, help="protein sequences (the middle residue is masked)")
    args = ap.parse_args(argv)
    from ..models.esm2 import EsmForMaskedLM
    from ..parallel.comm import init_distributed
    comm = init_distributed()
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    model = EsmForMaskedLM(ESM2_SIZES[args.size])
    if args.checkpoint:
        from ..io.checkpoint import Checkpoint
        ck = Checkpoint(args.checkpoint, prefix="")
        model.load_hf_state_dict({k: ck.raw(k) for k in ck.wm})
    else:
        model.init_weights(0)
    model = model.to(dev).eval()
    if comm.size > 1:
        from ..parallel.tensor_parallel import apply_esm_tp
        model = apply_esm_tp(model, comm)
    res = predict_masked_middle(model, args.sequences or DEFAULT_SEQUENCES, args.max_len)
    if comm.rank == 0:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
