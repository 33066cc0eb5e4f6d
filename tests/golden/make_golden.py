"""Generate the golden fixtures in this folder by running the reference's own eager PyTorch code on the CPU.

Run from the repository root, naming the reference checkout (read-only is fine) as the argument or in
``GRANITE_REFERENCE_ROOT``:

    python tests/golden/make_golden.py <reference root>

What it runs (all on CPU, PyTorch eager, imported unmodified from ``<reference>/script``):

* ``ConformerConvModule`` (``script/models/granite_speech_nar/conformer.py:158-189``) after ``fold_conv_bn_``
  (``script/models/granite_speech_nar/fold_bn.py:33``), plus the residual add of ``conformer.py:207``, in fp32
  (the CPU workload: B=1, T=256, seed 1001) and in bf16 (B=2, T=37, the load-time test-fire shape of
  ``conv_kernel.py:91-95``), with and without trimming each utterance to its length;
* the post-fold eager chain that ``granite::dwconv_silu`` replaces, ``F.silu(conv0(x))``
  (``conv_kernel.py:95-96``), and the fp64 golden of ``script/cuda_kernels/conv1d.py:135-138``;
* the GLU variant's eager chain ``F.silu(conv0(F.glu(x2, dim=1)))`` (``conv_kernel.py:91-92``);
* ``ConformerFeedForward`` (``conformer.py:23-40``) as the block applies it, ``x + 0.5 * ff(x)``
  (``conformer.py:205``, ``:208``), in fp32 and bf16 on the test-fire shape;
* ``ConformerAttention`` (``conformer.py:43-131``) as the block applies it, ``x + attn(x)`` (``conformer.py:206``),
  in fp32 and bf16, whole and with each utterance trimmed to a length;
* a whole ``ConformerBlock`` (``conformer.py:190-210``, BatchNorm folded by ``fold_conv_bn_``) in fp32 and bf16;
* the encoder's CTC heads: ``CTCEncoder.forward`` (``conformer.py:284-361``) with an identity projection and block,
  so the self-conditioning, pooling and BPE head run on the test input, then ``_collapse_ids_flat`` (``asr.py``);
* ``CTCEncoder.forward`` end to end with two Conformer blocks, from 160 input features to the BPE logits.

Inputs and parameters come from ``granite_conv_b200.synth`` (numpy PCG64 seeds), so the tests regenerate them
bit-for-bit and only the reference outputs are stored.  bf16 tensors are stored as uint16 bit patterns.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "granite-speech-4.1-2b-nar-turbo_b200"))
from granite_conv_b200 import synth  # noqa: E402


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _reference_module(ref_script: str):
    sys.path.insert(0, ref_script)
    from models.granite_speech_nar.conformer import ConformerConvModule  # noqa: E402
    from models.granite_speech_nar.config import EncoderConfig  # noqa: E402
    from models.granite_speech_nar.fold_bn import fold_conv_bn_  # noqa: E402
    return ConformerConvModule, EncoderConfig, fold_conv_bn_


def build_module(ConformerConvModule, EncoderConfig, fold_conv_bn_, p: synth.ConvModuleParams, dtype):
    m = ConformerConvModule(EncoderConfig())
    with torch.no_grad():
        m.norm.weight.copy_(torch.from_numpy(p.norm_weight))
        m.norm.bias.copy_(torch.from_numpy(p.norm_bias))
        m.up_conv.weight.copy_(torch.from_numpy(p.up_weight)[:, :, None])
        m.up_conv.bias.copy_(torch.from_numpy(p.up_bias))
        m.depth_conv.conv.weight.copy_(torch.from_numpy(p.dw_weight)[:, None, :])
        m.batch_norm.running_mean.copy_(torch.from_numpy(p.bn_mean))
        m.batch_norm.running_var.copy_(torch.from_numpy(p.bn_var))
        m.batch_norm.weight.copy_(torch.from_numpy(p.bn_weight))
        m.batch_norm.bias.copy_(torch.from_numpy(p.bn_bias))
        m.down_conv.weight.copy_(torch.from_numpy(p.down_weight)[:, :, None])
        m.down_conv.bias.copy_(torch.from_numpy(p.down_bias))
    m.eval()
    m = m.to(dtype)        # the fold casts back to the weight dtype, as in a bf16 model load
    assert fold_conv_bn_(m) == 1
    return m


@torch.no_grad()
def main(ref_root: str) -> None:
    torch.manual_seed(0)
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    CM, EC, fold = _reference_module(os.path.join(ref_root, "script"))
    out = {}

    # ---- fp32 CPU workload: B=1, T=256, seed 1001, no mask --------------------------------------------------
    p = synth.make_params(1001)
    x = synth.make_activations(1001 + 500, (1, 256, synth.D_MODEL))
    m = build_module(CM, EC, fold, p, torch.float32)
    xt = torch.from_numpy(x)
    y = (m(xt) + xt).numpy().astype(np.float64)
    flat = y.reshape(-1)
    idx = np.arange(0, flat.size, 61)
    np.savez_compressed(os.path.join(HERE, "module_fp32_b1t256.npz"),
                        row_sum=y.sum(axis=-1).reshape(-1), row_sumsq=(y * y).sum(axis=-1).reshape(-1),
                        sample_idx=idx.astype(np.int64), sample=flat[idx].astype(np.float32),
                        dw_weight_folded=m.depth_conv.conv.weight.detach().numpy()[:, 0, :].astype(np.float32),
                        dw_bias_folded=m.depth_conv.conv.bias.detach().numpy().astype(np.float32))
    out["module_fp32_b1t256"] = y.shape

    # ---- bf16 module, test-fire shape B=2, T=37; two weight scales; full and trimmed per utterance ---------
    for tag, seed, w_std in (("w002", 1003, 0.02), ("w006", 2003, 0.06)):
        p = synth.make_params(seed, w_std=w_std)
        x = synth.make_activations(seed + 500, (2, 37, synth.D_MODEL))
        m = build_module(CM, EC, fold, p, torch.bfloat16)
        xb = torch.from_numpy(x).to(torch.bfloat16)
        y_full = m(xb) + xb
        lengths = np.array([37, 23], dtype=np.int32)
        y_trim = [(m(xb[b:b + 1, :L]) + xb[b:b + 1, :L])[0] for b, L in enumerate(lengths)]
        np.savez_compressed(os.path.join(HERE, f"module_bf16_b2t37_{tag}.npz"),
                            full=_bits(y_full), lengths=lengths,
                            trimmed=np.concatenate([_bits(t) for t in y_trim], axis=0),
                            dw_weight_folded=_bits(m.depth_conv.conv.weight[:, 0, :]),
                            dw_bias_folded=_bits(m.depth_conv.conv.bias))
        out[f"module_bf16_{tag}"] = tuple(y_full.shape)

    # ---- granite::dwconv_silu and its GLU variant (channels-first, as the reference op takes them) ----------
    C, K = synth.D_INNER, synth.KERNEL
    w, b = synth.make_dw_weights(1002)
    conv0 = torch.nn.Conv1d(C, C, K, groups=C, bias=True, padding=K // 2)
    with torch.no_grad():
        conv0.weight.copy_(torch.from_numpy(w)[:, None, :])
        conv0.bias.copy_(torch.from_numpy(b))
    conv0 = conv0.to(torch.bfloat16)
    xs = synth.make_activations(1002 + 500, (1, C, 37))
    xb = torch.from_numpy(xs).to(torch.bfloat16)
    eager = F.silu(conv0(xb))
    golden64 = F.silu(F.conv1d(F.pad(xb.double(), (K // 2, K // 2)), conv0.weight.double(),
                               conv0.bias.double(), groups=C)).to(torch.bfloat16)
    x2 = synth.make_activations(1002 + 600, (1, 2 * C, 37))
    x2b = torch.from_numpy(x2).to(torch.bfloat16)
    eager_glu = F.silu(conv0(F.glu(x2b, dim=1)))
    np.savez_compressed(os.path.join(HERE, "dwconv_silu_b1c2048t37.npz"),
                        eager=_bits(eager), golden_fp64=_bits(golden64), eager_glu=_bits(eager_glu))
    out["dwconv_silu"] = tuple(eager.shape)

    # ---- fp64 golden on the conv1d.py self-test length T=261: statistics only ------------------------------
    xs = synth.make_activations(1002 + 700, (1, C, 261))
    xb = torch.from_numpy(xs).to(torch.bfloat16)
    g = F.silu(F.conv1d(F.pad(xb.double(), (K // 2, K // 2)), conv0.weight.double(), conv0.bias.double(),
                        groups=C)).to(torch.bfloat16).double().numpy()
    np.savez_compressed(os.path.join(HERE, "dwconv_silu_stats_c2048t261.npz"),
                        chan_sum=g.sum(axis=-1).reshape(-1), chan_sumsq=(g * g).sum(axis=-1).reshape(-1))
    out["dwconv_silu_stats"] = g.shape

    # ---- feed-forward half of the block: x + 0.5 * ConformerFeedForward(x) (conformer.py:23-40, :205, :208) ------
    from models.granite_speech_nar.conformer import ConformerFeedForward  # noqa: E402
    for tag, seed, w_std in (("w002", 1101, 0.02), ("w006", 1102, 0.06)):
        fp = synth.make_ff_params(seed, w_std=w_std)
        ff = ConformerFeedForward(EC())
        with torch.no_grad():
            ff.pre_norm.weight.copy_(torch.from_numpy(fp.norm_weight))
            ff.pre_norm.bias.copy_(torch.from_numpy(fp.norm_bias))
            ff.up_proj.weight.copy_(torch.from_numpy(fp.up_weight))
            ff.up_proj.bias.copy_(torch.from_numpy(fp.up_bias))
            ff.down_proj.weight.copy_(torch.from_numpy(fp.down_weight))
            ff.down_proj.bias.copy_(torch.from_numpy(fp.down_bias))
        ff.eval()
        x = synth.make_activations(seed + 500, (2, 37, synth.D_MODEL))
        # fp32 and bf16 (a bf16 model load) on the test-fire shape
        xf = torch.from_numpy(x)
        y32 = (0.5 * ff(xf) + xf).numpy()
        ffb = ff.to(torch.bfloat16)
        xb = xf.to(torch.bfloat16)
        yb = 0.5 * ffb(xb) + xb
        np.savez_compressed(os.path.join(HERE, f"ff_half_b2t37_{tag}.npz"), bf16=_bits(yb), fp32=y32)
        out[f"ff_half_{tag}"] = tuple(yb.shape)

    # ---- attention step of the block: x + ConformerAttention(x) (conformer.py:43-131, :206) --------------------
    # bf16 (a bf16 model load) on CPU, where the attention runs the MATH backend; T = 37 (one partial block) and
    # T = 237 (a full block and a partial one), with the encoder's attention_dists (conformer.py:254-262)
    from models.granite_speech_nar.conformer import ConformerAttention  # noqa: E402
    for tag, seed, w_std, T in (("w002_t237", 1201, 0.02, 237), ("w006_t37", 1202, 0.06, 37),
                                ("w006_t237", 1203, 0.06, 237)):
        ap = synth.make_attn_params(seed, w_std=w_std)
        at = ConformerAttention(EC())
        with torch.no_grad():
            at.pre_norm.weight.copy_(torch.from_numpy(ap.norm_weight))
            at.pre_norm.bias.copy_(torch.from_numpy(ap.norm_bias))
            at.to_q.weight.copy_(torch.from_numpy(ap.q_weight))
            at.to_kv.weight.copy_(torch.from_numpy(ap.kv_weight))
            at.to_out.weight.copy_(torch.from_numpy(ap.out_weight))
            at.to_out.bias.copy_(torch.from_numpy(ap.out_bias))
            at.rel_pos_emb.weight.copy_(torch.from_numpy(ap.rel_pos))
        at.eval()
        cs = at.context_size
        seq = torch.arange(cs)
        dists = torch.clamp(seq.view(-1, 1) - seq.view(1, -1), -cs, cs) + at.max_pos_emb
        x = synth.make_activations(seed + 500, (2, T, synth.D_MODEL))
        xf = torch.from_numpy(x)
        y32 = (at(xf, attention_dists=dists) + xf).numpy()
        atb = at.to(torch.bfloat16)
        xb = xf.to(torch.bfloat16)
        yb = atb(xb, attention_dists=dists) + xb
        lengths = np.array([T, max(1, (2 * T) // 3)], dtype=np.int32)
        y_trim = [(atb(xb[b:b + 1, :L], attention_dists=dists) + xb[b:b + 1, :L])[0] for b, L in enumerate(lengths)]
        np.savez_compressed(os.path.join(HERE, f"attn_b2_{tag}.npz"), bf16=_bits(yb), fp32=y32, lengths=lengths,
                            trimmed=np.concatenate([_bits(t) for t in y_trim], axis=0))
        out[f"attn_{tag}"] = tuple(yb.shape)

    # ---- whole Conformer block: FF/2, attention, conv, FF/2, post norm (conformer.py:190-210) ----------------------
    from models.granite_speech_nar.conformer import ConformerBlock  # noqa: E402
    bp = synth.make_block_params(1301, w_std=0.02)
    blk = ConformerBlock(EC())
    _load_block(blk, bp)
    blk.eval()
    _block_golden(blk, bp, fold, out)
    _ctc_goldens(EC, out)
    _encoder_golden(EC, fold, out)

    for k, v in out.items():
        print(f"{k}: {v}")


def _load_block(blk, bp):
    with torch.no_grad():
        for name, fp in (("ff1", bp.ff1), ("ff2", bp.ff2)):
            ff = getattr(blk, name)
            ff.pre_norm.weight.copy_(torch.from_numpy(fp.norm_weight))
            ff.pre_norm.bias.copy_(torch.from_numpy(fp.norm_bias))
            ff.up_proj.weight.copy_(torch.from_numpy(fp.up_weight))
            ff.up_proj.bias.copy_(torch.from_numpy(fp.up_bias))
            ff.down_proj.weight.copy_(torch.from_numpy(fp.down_weight))
            ff.down_proj.bias.copy_(torch.from_numpy(fp.down_bias))
        ap = bp.attn
        blk.attn.pre_norm.weight.copy_(torch.from_numpy(ap.norm_weight))
        blk.attn.pre_norm.bias.copy_(torch.from_numpy(ap.norm_bias))
        blk.attn.to_q.weight.copy_(torch.from_numpy(ap.q_weight))
        blk.attn.to_kv.weight.copy_(torch.from_numpy(ap.kv_weight))
        blk.attn.to_out.weight.copy_(torch.from_numpy(ap.out_weight))
        blk.attn.to_out.bias.copy_(torch.from_numpy(ap.out_bias))
        blk.attn.rel_pos_emb.weight.copy_(torch.from_numpy(ap.rel_pos))
        cp = bp.conv
        m = blk.conv
        m.norm.weight.copy_(torch.from_numpy(cp.norm_weight))
        m.norm.bias.copy_(torch.from_numpy(cp.norm_bias))
        m.up_conv.weight.copy_(torch.from_numpy(cp.up_weight)[:, :, None])
        m.up_conv.bias.copy_(torch.from_numpy(cp.up_bias))
        m.depth_conv.conv.weight.copy_(torch.from_numpy(cp.dw_weight)[:, None, :])
        m.batch_norm.running_mean.copy_(torch.from_numpy(cp.bn_mean))
        m.batch_norm.running_var.copy_(torch.from_numpy(cp.bn_var))
        m.batch_norm.weight.copy_(torch.from_numpy(cp.bn_weight))
        m.batch_norm.bias.copy_(torch.from_numpy(cp.bn_bias))
        m.down_conv.weight.copy_(torch.from_numpy(cp.down_weight)[:, :, None])
        m.down_conv.bias.copy_(torch.from_numpy(cp.down_bias))
        blk.post_norm.weight.copy_(torch.from_numpy(bp.post_norm_weight))
        blk.post_norm.bias.copy_(torch.from_numpy(bp.post_norm_bias))


def _block_golden(blk, bp, fold, out):
    from models.granite_speech_nar.conformer import ConformerBlock  # noqa: E402
    from models.granite_speech_nar.config import EncoderConfig as EC  # noqa: E402
    cs = blk.attn.context_size
    seq = torch.arange(cs)
    dists = torch.clamp(seq.view(-1, 1) - seq.view(1, -1), -cs, cs) + blk.attn.max_pos_emb
    T = 237
    x = synth.make_activations(1801, (2, T, synth.D_MODEL))
    xf = torch.from_numpy(x)
    b32 = ConformerBlock(EC())
    b32.load_state_dict(blk.state_dict())
    b32.eval()
    assert fold(b32) == 1
    y32 = b32(xf, attention_dists=dists).numpy()
    bb = blk.to(torch.bfloat16)
    assert fold(bb) == 1
    xb = xf.to(torch.bfloat16)
    yb = bb(xb, attention_dists=dists)
    lengths = np.array([T, 150], dtype=np.int32)
    y_trim = [bb(xb[b:b + 1, :L], attention_dists=dists)[0] for b, L in enumerate(lengths)]
    np.savez_compressed(os.path.join(HERE, "block_b2_t237_w002.npz"), bf16=_bits(yb), fp32=y32, lengths=lengths,
                        trimmed=np.concatenate([_bits(t) for t in y_trim], axis=0))
    out["block_w002_t237"] = tuple(yb.shape)


def _ctc_goldens(EC, out):
    # ---- CTC heads: CTCEncoder.forward's self-conditioning, pooling and BPE head (conformer.py:284-361), and the
    # CTC collapse (asr.py:76-102).  The encoder gets an identity input projection and one identity block, so its
    # hidden state is the test input; vocabulary 2048 (blank 7) to keep the fixture small.
    from models.granite_speech_nar.conformer import CTCEncoder  # noqa: E402
    from models.granite_speech_nar.asr import _collapse_ids_flat  # noqa: E402

    class _Identity(torch.nn.Module):
        def forward(self, x, **kwargs):
            return x

    V, blank = 2048, 7
    cp = synth.make_ctc_params(1401, vocab=V, blank_id=blank)
    cfg = EC(input_dim=synth.D_MODEL, num_layers=1, self_conditioning_layer=1, bpe_output_dim=V, blank_token_id=blank)
    enc = CTCEncoder(cfg)
    enc.layers = torch.nn.ModuleList([_Identity()])
    with torch.no_grad():
        enc.input_linear.weight.copy_(torch.eye(synth.D_MODEL))
        enc.input_linear.bias.zero_()
        enc.out.weight.copy_(torch.from_numpy(cp.out_weight))
        enc.out.bias.copy_(torch.from_numpy(cp.out_bias))
        enc.out_mid.weight.copy_(torch.from_numpy(cp.mid_weight))
        enc.out_mid.bias.copy_(torch.from_numpy(cp.mid_bias))
        enc.out_bpe.weight.copy_(torch.from_numpy(cp.bpe_weight))
        enc.out_bpe.bias.copy_(torch.from_numpy(cp.bpe_bias))
    enc.eval()
    encb = enc.to(torch.bfloat16)
    T = 37
    x = synth.make_activations(1901, (2, T, synth.D_MODEL))
    xb = torch.from_numpy(x).to(torch.bfloat16)
    res = {}
    lengths = np.array([T, 23], dtype=np.int32)
    for tag, batch in (("whole", [(0, T), (1, T)]), ("trimmed", [(b, int(L)) for b, L in enumerate(lengths)])):
        ids_all, logits_all, hid_all, seg = [], [], [], []
        for b, L in batch:
            o = encb(xb[b:b + 1, :L], attention_mask=torch.ones((1, L), dtype=torch.bool),
                     output_hidden_states=False)
            ids_all.append(o.logits.argmax(-1))
            logits_all.append(o.logits)
            hid_all.append(o.last_hidden_state[0])
            seg.append(int(o.logits.shape[0]))
        flat = torch.cat(ids_all)
        toks, counts, _ = _collapse_ids_flat(flat, seg, blank)
        res[f"{tag}_ids"] = flat.numpy().astype(np.int32)
        res[f"{tag}_logits"] = _bits(torch.cat(logits_all))
        res[f"{tag}_hidden"] = np.concatenate([_bits(h) for h in hid_all], axis=0)
        res[f"{tag}_tokens"] = (torch.cat(toks).numpy().astype(np.int32) if sum(counts) else np.zeros(0, np.int32))
        res[f"{tag}_counts"] = np.array(counts, dtype=np.int32)
        res[f"{tag}_segments"] = np.array(seg, dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "ctc_heads_b2_t37_v2048.npz"), lengths=lengths, **res)
    out["ctc_heads"] = tuple(res["whole_ids"].shape)


def _encoder_golden(EC, fold, out):
    """CTCEncoder.forward end to end (conformer.py:284-361): input projection from 160 features, two Conformer blocks,
    the self-conditioning after block 1, the BPE head; BatchNorm folded as the reference loader does; bf16."""
    from models.granite_speech_nar.conformer import CTCEncoder  # noqa: E402
    from models.granite_speech_nar.asr import _collapse_ids_flat  # noqa: E402
    V, blank = 2048, 7
    cfg = EC(num_layers=2, self_conditioning_layer=1, bpe_output_dim=V, blank_token_id=blank)
    enc = CTCEncoder(cfg)
    w_in, b_in = synth.make_input_params(1501)
    cp = synth.make_ctc_params(1502, vocab=V, blank_id=blank)
    with torch.no_grad():
        enc.input_linear.weight.copy_(torch.from_numpy(w_in))
        enc.input_linear.bias.copy_(torch.from_numpy(b_in))
        for i, layer in enumerate(enc.layers):
            _load_block(layer, synth.make_block_params(1503 + i, w_std=0.02))
        enc.out.weight.copy_(torch.from_numpy(cp.out_weight))
        enc.out.bias.copy_(torch.from_numpy(cp.out_bias))
        enc.out_mid.weight.copy_(torch.from_numpy(cp.mid_weight))
        enc.out_mid.bias.copy_(torch.from_numpy(cp.mid_bias))
        enc.out_bpe.weight.copy_(torch.from_numpy(cp.bpe_weight))
        enc.out_bpe.bias.copy_(torch.from_numpy(cp.bpe_bias))
    enc.eval()
    enc = enc.to(torch.bfloat16)
    assert fold(enc) == 2
    T = 237
    feats = synth.make_activations(1601, (2, T, synth.INPUT_DIM))
    fb = torch.from_numpy(feats).to(torch.bfloat16)
    res = {}
    lengths = np.array([T, 150], dtype=np.int32)
    for tag, batch in (("whole", [(0, T), (1, T)]), ("trimmed", [(b, int(L)) for b, L in enumerate(lengths)])):
        ids_all, logits_all, hid_all, seg = [], [], [], []
        for b, L in batch:
            o = enc(fb[b:b + 1, :L], attention_mask=torch.ones((1, L), dtype=torch.bool), output_hidden_states=False)
            ids_all.append(o.logits.argmax(-1))
            logits_all.append(o.logits)
            hid_all.append(o.last_hidden_state[0])
            seg.append(int(o.logits.shape[0]))
        flat = torch.cat(ids_all)
        toks, counts, _ = _collapse_ids_flat(flat, seg, blank)
        res[f"{tag}_ids"] = flat.numpy().astype(np.int32)
        res[f"{tag}_logits"] = _bits(torch.cat(logits_all))
        res[f"{tag}_hidden"] = np.concatenate([_bits(h) for h in hid_all], axis=0)
        res[f"{tag}_tokens"] = (torch.cat(toks).numpy().astype(np.int32) if sum(counts) else np.zeros(0, np.int32))
        res[f"{tag}_counts"] = np.array(counts, dtype=np.int32)
        res[f"{tag}_segments"] = np.array(seg, dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "encoder_l2_b2_t237_v2048.npz"), lengths=lengths, **res)
    out["encoder_l2"] = tuple(res["whole_ids"].shape)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GRANITE_REFERENCE_ROOT", "")
    if not root:
        sys.exit("usage: make_golden.py <reference root>  (or set GRANITE_REFERENCE_ROOT)")
    main(root)
