"""The detector after the stem on B200 kernels: ``SarbonDetector.forward(None, p8=...)``.

Reference: Bahrombekk/Sarbon ``sarbon/models/sarbon_det.py`` -- ``DenseCore`` (:118-155), the
encoder's query selection (:306-321) and the decoder with its box heads (:336-366), run by
``SarbonVideo._run_det`` under ``torch.autocast(float16)`` (sarbon/inference/video.py:116-118).

``B200Detector(det, batch, h8, w8)`` takes the reference's own detector module (its weights),
folds every BatchNorm into fp16 weight matrices once, and runs inference on the cached p8
with the kernels of ``libsarbon_sparse.so`` only:

* every Conv2d / Linear (3x3 stride 1 and 2, 1x1 over two concatenated maps, the MLP heads)
  is one ``sb_gemm_conv`` launch (tcgen05 implicit GEMM) with its bias, residual and ReLU /
  GELU fused;
* LayerNorms (``sb_layernorm``), the depthwise half of ``fuse()`` (``sb_dwconv3x3``), the
  nearest upsampling (``sb_upsample2x``), both attentions (``sb_attention``), the top-K
  query selection (``sb_topk_rows``), the deformable sampling with its softmax and
  box-relative locations (``sb_deform_sample``) and the box heads (``sb_box_enc``,
  ``sb_box_dec``) are one kernel each;
* the three output levels are written straight into the decoder's concatenated memory
  (no torch.cat), and the whole forward can be replayed as one CUDA graph (``capture``).

Values follow the reference's autocast dtype flow: fp16 products with fp32 accumulation,
LayerNorm / softmax in fp32, the fp32 residual stream of the decoder, fp16 box arithmetic
where the reference box is fp16.  Differences from the reference's forward, all without
effect on its outputs: rows outside the valid anchor area are not zeroed before
``enc_proj`` (they never reach the outputs: the query selection masks them and only
selected rows are gathered), the encoder's box MLP runs on the selected rows only, and the
training-only parts (denoising queries, auxiliary per-layer outputs) and track queries are
not built.  Supported configuration: ``fusion="concat"``, ``block_type="res"``,
``act="relu"`` (the reference's defaults and every size in ``SIZES``).
"""
from __future__ import annotations

import torch

from . import det_ops as ops


def _fold_conv_bn(conv, bn):
    """Conv2d (no bias) + BatchNorm2d (eval) -> fp32 weight [cout, cin, kh, kw], bias [cout]."""
    scale = bn.weight.detach().float() / torch.sqrt(bn.running_var.detach().float() + bn.eps)
    w = conv.weight.detach().float() * scale.view(-1, 1, 1, 1)
    b = bn.bias.detach().float() - bn.running_mean.detach().float() * scale
    if conv.bias is not None:
        b = b + conv.bias.detach().float() * scale
    return w, b


def _conv_mat(w):
    """[cout, cin, kh, kw] -> fp16 [cout, kh*kw*cin] with columns (tap = ky*3 + kx, channel)."""
    return w.permute(0, 2, 3, 1).reshape(w.shape[0], -1).half().contiguous()


def _lin(m, pad_k=None):
    w = m.weight.detach().float()
    if pad_k is not None and w.shape[1] < pad_k:
        w = torch.cat([w, w.new_zeros(w.shape[0], pad_k - w.shape[1])], 1)
    b = m.bias.detach().float().contiguous() if m.bias is not None else None
    return w.half().contiguous(), b


def sincos_2d(h, w, dim, device, temperature=10000.0):
    """2-D sine-cosine position table [h*w, dim] (the reference's sincos_2d, sarbon_det.py:109-115)."""
    y, x = torch.meshgrid(torch.arange(h, device=device, dtype=torch.float32),
                          torch.arange(w, device=device, dtype=torch.float32), indexing="ij")
    d = dim // 4
    omega = 1.0 / temperature ** (torch.arange(d, device=device, dtype=torch.float32) / d)
    ox, oy = x.flatten()[:, None] * omega, y.flatten()[:, None] * omega
    return torch.cat([ox.sin(), ox.cos(), oy.sin(), oy.cos()], 1)


def anchors_of(shapes, device):
    """Cell-centre anchors in logit space and their validity (sarbon_det.py:276-289)."""
    out = []
    for lvl, (h, w) in enumerate(shapes):
        y, x = torch.meshgrid(torch.arange(h, device=device), torch.arange(w, device=device), indexing="ij")
        xy = torch.stack([(x + 0.5) / w, (y + 0.5) / h], -1).view(-1, 2)
        out.append(torch.cat([xy, torch.full_like(xy, 0.05 * 2.0 ** lvl)], -1))
    a = torch.cat(out)
    valid = ((a > 0.01) & (a < 0.99)).all(-1)
    a = a.clamp(1e-5, 1 - 1e-5)
    logit = torch.log(a / (1 - a)).masked_fill(~valid[:, None], float("inf"))
    return logit.half().contiguous(), valid.to(torch.uint8).contiguous()


class B200Detector:
    """Inference of a reference ``SarbonDetector`` from p8 on; see the module docstring."""

    def __init__(self, det, batch: int, h8: int, w8: int, device="cuda"):
        cfg = det.cfg
        if cfg.fusion != "concat" or cfg.block_type != "res" or cfg.act != "relu":
            raise NotImplementedError("B200Detector supports fusion='concat', block_type='res', act='relu'")
        dev = torch.device(device)
        self.dev, self.B, self.cfg = dev, batch, cfg
        d = cfg.hidden
        self.d, self.heads, self.points, self.K = d, cfg.heads, cfg.points, cfg.queries
        self.nc = det.num_classes
        h16, w16 = (h8 - 1) // 2 + 1, (w8 - 1) // 2 + 1
        h32, w32 = (h16 - 1) // 2 + 1, (w16 - 1) // 2 + 1
        if 2 * h32 != h16 or 2 * w32 != w16 or 2 * h16 != h8 or 2 * w16 != w8:
            raise ValueError("the p8 size must halve exactly twice (the reference's top-down cat needs it)")
        self.shapes = [(h8, w8), (h16, w16), (h32, w32)]
        self.S = sum(h * w for h, w in self.shapes)
        self.level_off = [0, h8 * w8, h8 * w8 + h16 * w16]
        core = det.core
        c8 = core.in8[0].in_channels
        self.c8 = c8

        def cba(m):  # conv_bn_act -> (fp16 matrix, fp32 bias)
            w, b = _fold_conv_bn(m[0], m[1])
            return _conv_mat(w).to(dev), b.to(dev)

        def res(m):  # Res block
            return cba(m.body[0]), cba(m.body[1])

        def fuse(m):  # 1x1 + BN + ReLU, dw3x3 + BN + ReLU
            w1, b1 = _fold_conv_bn(m[0], m[1])
            w2, b2 = _fold_conv_bn(m[3], m[4])
            return (_conv_mat(w1).to(dev), b1.to(dev),
                    w2.view(w2.shape[0], 9).t().contiguous().to(dev), b2.contiguous().to(dev))

        with torch.no_grad():
            self.w_to16 = cba(core.to16[0])
            self.w_res16 = [res(core.to16[1]), res(core.to16[2])]
            self.w_to32 = cba(core.to32[0])
            self.w_res32 = [res(core.to32[1])]
            self.w_in = [cba(m) for m in (core.in8, core.in16, core.in32)]
            a = core.aifi
            self.aifi = dict(
                qkv=(a.self_attn.in_proj_weight.detach().half().contiguous().to(dev),
                     a.self_attn.in_proj_bias.detach().float().contiguous().to(dev)),
                out=[t.to(dev) for t in _lin(a.self_attn.out_proj)],
                l1=[t.to(dev) for t in _lin(a.linear1)], l2=[t.to(dev) for t in _lin(a.linear2)],
                n1=(a.norm1.weight.detach().float().to(dev), a.norm1.bias.detach().float().to(dev), a.norm1.eps),
                n2=(a.norm2.weight.detach().float().to(dev), a.norm2.bias.detach().float().to(dev), a.norm2.eps))
            self.heads_aifi = a.self_attn.num_heads
            self.w_td16, self.w_td8 = fuse(core.td16), fuse(core.td8)
            self.w_bu16, self.w_bu32 = fuse(core.bu16), fuse(core.bu32)
            self.w_down8, self.w_down16 = cba(core.down8), cba(core.down16)
            self.pos32 = sincos_2d(h32, w32, d, dev).half().contiguous()
            # encoder heads
            self.w_encp = [t.to(dev) for t in _lin(det.enc_proj[0])]
            ln = det.enc_proj[1]
            self.n_enc = (ln.weight.detach().float().to(dev), ln.bias.detach().float().to(dev), ln.eps)
            self.w_enc_cls = [t.to(dev) for t in _lin(det.enc_cls)]
            self.w_enc_box = [[t.to(dev) for t in _lin(det.enc_box[i])] for i in (0, 2, 4)]
            self.anchors, self.valid = anchors_of(self.shapes, dev)
            # decoder
            self.w_qpos = [[t.to(dev) for t in _lin(det.query_pos[0], pad_k=64)],
                           [t.to(dev) for t in _lin(det.query_pos[2])]]
            self.w_layers = []
            for L in det.layers:
                sa, cr = L.self_attn, L.cross
                wi, bi = sa.in_proj_weight.detach(), sa.in_proj_bias.detach()
                off_w = torch.cat([cr.offsets.weight.detach(), cr.attn.weight.detach()], 0)
                off_b = torch.cat([cr.offsets.bias.detach(), cr.attn.bias.detach()], 0)
                self.w_layers.append(dict(
                    qk=(wi[:2 * d].half().contiguous().to(dev), bi[:2 * d].float().contiguous().to(dev)),
                    v=(wi[2 * d:].half().contiguous().to(dev), bi[2 * d:].float().contiguous().to(dev)),
                    o=[t.to(dev) for t in _lin(sa.out_proj)],
                    value=_lin(cr.value_proj),
                    offatt=(off_w.half().contiguous().to(dev), off_b.float().contiguous().to(dev)),
                    n_off=cr.offsets.out_features,
                    cout=[t.to(dev) for t in _lin(cr.out_proj)],
                    f1=[t.to(dev) for t in _lin(L.ffn[0])], f2=[t.to(dev) for t in _lin(L.ffn[2])],
                    n=[(n.weight.detach().float().to(dev), n.bias.detach().float().to(dev), n.eps)
                       for n in (L.n1, L.n2, L.n3)]))
                if cr.h != self.heads or cr.p != self.points or cr.l != 3:
                    raise NotImplementedError("MSDeformAttn with 3 levels and the config's heads / points")
            # every layer's value projection reads the same memory: one GEMM with the layers'
            # weights stacked along N (layer i's value = columns i*d .. (i+1)*d of its output)
            vals = [w.pop("value") for w in self.w_layers]
            self.w_value = (torch.cat([v[0] for v in vals], 0).contiguous().to(dev),
                            torch.cat([v[1] for v in vals], 0).contiguous().to(dev))
            self.w_cls = [[t.to(dev) for t in _lin(h)] for h in det.cls_heads]
            self.w_pre = [[t.to(dev) for t in _lin(det.pre_box[i])] for i in (0, 2, 4)]
            self.w_corner = [[[t.to(dev) for t in _lin(h[i])] for i in (0, 2, 4)] for h in det.corner_heads]
            self.w_id = [[t.to(dev) for t in _lin(det.id_head[i])] for i in (0, 2)]
            self.project = det.project.detach().float().contiguous().to(dev)
            self.reg_scale = float(cfg.reg_scale)
        self._alloc()
        self.graph = None
        self._graph_in = None

    # ------------------------------------------------------------ buffers
    def _alloc(self):
        B, d, K, S, dev = self.B, self.d, self.K, self.S, self.dev
        (h8, w8), (h16, w16), (h32, w32) = self.shapes
        f16, f32 = dict(device=dev, dtype=torch.float16), dict(device=dev, dtype=torch.float32)
        e = lambda *s, **k: torch.empty(*s, **k)  # noqa: E731
        self.mem = e(B, S, d, **f16)
        self.b16 = [e(B, h16, w16, d, **f16) for _ in range(3)]
        self.b32 = [e(B, h32, w32, d, **f16) for _ in range(3)]
        self.x8 = e(B, h8, w8, d, **f16)
        self.x16 = e(B, h16, w16, d, **f16)
        self.x32 = e(B, h32, w32, d, **f16)
        T = h32 * w32
        self.T = T
        self.t_pos = e(B, T, d, **f16)
        self.qkv = e(B, T, 3 * d, **f16)
        self.att_t = e(B, T, d, **f16)
        self.sa_t = e(B, T, d, **f16)
        self.ln1_32 = e(B, T, d, **f32)
        self.ln1_16 = e(B, T, d, **f16)
        self.ffn_t = e(B, T, self.aifi["l1"][0].shape[0], **f16)
        self.ffn2_t = e(B, T, d, **f16)
        self.x32b = e(B, h32, w32, d, **f16)  # aifi(t + pos) - pos
        self.up16 = e(B, h16, w16, d, **f16)
        self.f16a = e(B, h16, w16, d, **f16)
        self.t16 = e(B, h16, w16, d, **f16)
        self.up8 = e(B, h8, w8, d, **f16)
        self.f8a = e(B, h8, w8, d, **f16)
        self.d8 = e(B, h16, w16, d, **f16)
        self.f16b = e(B, h16, w16, d, **f16)
        self.d16 = e(B, h32, w32, d, **f16)
        self.f32b = e(B, h32, w32, d, **f16)
        # encoder
        self.enc_lin = e(B, S, d, **f16)
        self.enc16 = e(B, S, d, **f16)
        self.enc_sel = e(B, K, d, **f16)  # enc_proj rows of the selected queries, before the LayerNorm
        self.enc_logits = e(B, S, self.nc, **f16)
        self.top = e(B, K, device=dev, dtype=torch.int32)
        self.tgt32 = [e(B, K, d, **f32), e(B, K, d, **f32)]
        self.mid32 = e(B, K, d, **f32)  # the residual stream between a layer's LayerNorms
        self.tgt16 = e(B, K, d, **f16)
        self.h1 = e(B, K, d, **f16)
        self.h2 = e(B, K, d, **f16)
        self.encbox = e(B, K, 4, **f16)
        self.ref16 = e(B, K, 4, **f16)
        self.qin = torch.zeros(B, K, 64, **f16)
        self.enc_logits_sel = e(B, K, self.nc, **f32)
        # decoder
        self.qp1 = e(B, K, self.w_qpos[0][0].shape[0], **f16)
        self.pos = e(B, K, d, **f16)
        self.q16 = e(B, K, d, **f16)
        self.qk = e(B, K, 2 * d, **f16)
        self.vv = e(B, K, d, **f16)
        self.att_q = e(B, K, d, **f16)
        self.sa_q = e(B, K, d, **f16)
        self.qc16 = e(B, K, d, **f16)
        self.value = e(B, S, len(self.w_layers) * d, **f16)  # all layers' values of the memory
        n_oa = self.w_layers[0]["offatt"][0].shape[0]
        self.offatt = e(B, K, n_oa, **f16)
        self.samp = e(B, K, d, **f16)
        self.cross = e(B, K, d, **f16)
        self.ffn_in = e(B, K, d, **f16)
        self.ffn_q = e(B, K, self.w_layers[0]["f1"][0].shape[0], **f16)
        self.ffn2_q = e(B, K, d, **f16)
        self.head_in = e(B, K, d, **f16)
        self.pb = e(B, K, 4, **f16)
        self.head = e(B, K, self.w_corner[0][2][0].shape[0], **f16)
        self.corners = e(B, K, self.w_corner[0][2][0].shape[0], **f16)
        self.ref_init = e(B, K, 4, **f32)
        self.box = e(B, K, 4, **f32)
        self.logits = e(B, K, self.nc, **f16)
        self.idh = e(B, K, self.w_id[0][0].shape[0], **f16)
        self.idv = e(B, K, self.w_id[1][0].shape[0], **f16)
        self.id_embed = e(B, K, self.w_id[1][0].shape[0], **f32)
        self.force_top = None

    # ------------------------------------------------------------ pieces
    def _fuse(self, w, a, b, tmp, out):
        ops.gemm_conv([a, b], w[0], w[1], act="relu", out=tmp)
        ops.dwconv3x3(tmp, w[2], w[3], relu=True, out=out)

    def _mlp(self, ws, x, hidden, out, last_act=None):
        h = x
        for i, (w, b) in enumerate(ws[:-1]):
            ops.gemm_conv(h.view(-1, h.shape[-1]), w, b, act="relu", out=hidden[i].view(-1, w.shape[0]))
            h = hidden[i]
        w, b = ws[-1]
        ops.gemm_conv(h.view(-1, h.shape[-1]), w, b, act=last_act, out=out.view(-1, w.shape[0]))
        return out

    def level(self, i):
        """Level i of the memory as an NHWC view [B, h, w, d]."""
        h, w = self.shapes[i]
        o = self.level_off[i]
        return self.mem[:, o:o + h * w].view(self.B, h, w, self.d)

    def core(self, x8in):
        """DenseCore (sarbon_det.py:141-155) into the memory's three levels."""
        B, d = self.B, self.d
        g = ops.gemm_conv
        # to16, to32 with their Res units
        g(x8in, *self.w_to16, act="relu", taps=9, stride=2, out=self.b16[0])
        cur = self.b16[0]
        for k, (c1, c2) in enumerate(self.w_res16):
            g(cur, *c1, act="relu", taps=9, out=self.b16[1])
            nxt = self.b16[2] if cur is self.b16[0] else self.b16[0]
            g(self.b16[1], *c2, act="relu", taps=9, res=cur, out=nxt)
            cur = nxt
        p16 = cur
        g(p16, *self.w_to32, act="relu", taps=9, stride=2, out=self.b32[0])
        cur = self.b32[0]
        for c1, c2 in self.w_res32:
            g(cur, *c1, act="relu", taps=9, out=self.b32[1])
            nxt = self.b32[2] if cur is self.b32[0] else self.b32[0]
            g(self.b32[1], *c2, act="relu", taps=9, res=cur, out=nxt)
            cur = nxt
        p32 = cur
        g(x8in, *self.w_in[0], out=self.x8)
        g(p16, *self.w_in[1], out=self.x16)
        g(p32, *self.w_in[2], out=self.x32)
        # AIFI on the stride-32 tokens: x = t + pos; x = n1(x + sa(x)); x = n2(x + ffn(x)); - pos
        T, a = self.T, self.aifi
        t = self.x32.view(B, T, d)
        ops.add_rows(t, self.pos32, self.t_pos, period=T)
        g(self.t_pos.view(B * T, d), *a["qkv"], out=self.qkv.view(B * T, 3 * d))
        ops.attention(self.qkv[..., :d], self.qkv[..., d:2 * d], self.qkv[..., 2 * d:], self.heads_aifi, out=self.att_t)
        g(self.att_t.view(B * T, d), *a["out"], out=self.sa_t.view(B * T, d))
        ops.layernorm(self.t_pos, a["n1"][0], a["n1"][1], a["n1"][2], b=self.sa_t, y32=self.ln1_32, y16=self.ln1_16)
        g(self.ln1_16.view(B * T, d), *a["l1"], act="gelu", out=self.ffn_t.view(B * T, -1))
        g(self.ffn_t.view(B * T, -1), *a["l2"], out=self.ffn2_t.view(B * T, d))
        ops.layernorm(self.ln1_32, a["n2"][0], a["n2"][1], a["n2"][2], b=self.ffn2_t, pos=self.pos32, sign=-1.0,
                      yp16=self.x32b.view(B, T, d), period=T)
        # top-down and bottom-up fusion; the outputs land in the memory levels
        ops.upsample2x(self.x32b, out=self.up16)
        self._fuse(self.w_td16, self.x16, self.up16, self.f16a, self.t16)
        ops.upsample2x(self.t16, out=self.up8)
        o8, o16, o32 = self.level(0), self.level(1), self.level(2)
        self._fuse(self.w_td8, self.x8, self.up8, self.f8a, o8)
        g(o8, *self.w_down8, act="relu", taps=9, stride=2, out=self.d8)
        self._fuse(self.w_bu16, self.t16, self.d8, self.f16b, o16)
        g(o16, *self.w_down16, act="relu", taps=9, stride=2, out=self.d16)
        self._fuse(self.w_bu32, self.x32b, self.d16, self.f32b, o32)

    def encoder(self):
        """Query selection (sarbon_det.py:306-321)."""
        B, S, d, K = self.B, self.S, self.d, self.K
        g = ops.gemm_conv
        g(self.mem.view(B * S, d), *self.w_encp, out=self.enc_lin.view(B * S, d))
        # fp16 rows for the class head; the fp32 rows are needed for the selected queries only,
        # whose LayerNorm (row-local, the same kernel) is recomputed after the selection
        ops.layernorm(self.enc_lin, *self.n_enc, y16=self.enc16)
        g(self.enc16.view(B * S, d), *self.w_enc_cls, out=self.enc_logits.view(B * S, self.nc))
        if self.force_top is not None:
            self.top.copy_(self.force_top)
        else:
            ops.topk_rows(self.enc_logits, K, self.valid, out=self.top)
        ops.gather_rows(self.enc_lin, self.top, o16=self.enc_sel)
        ops.layernorm(self.enc_sel, *self.n_enc, y32=self.tgt32[0], y16=self.tgt16)
        ops.gather_rows(self.enc_logits, self.top, o32=self.enc_logits_sel)
        self._mlp(self.w_enc_box, self.tgt16, [self.h1, self.h2], self.encbox)
        ops.box_enc(self.encbox.view(B * K, 4), self.anchors, self.top, self.ref16, self.qin.view(B * K, 64))

    def decoder(self):
        """Decoder layers and box heads (sarbon_det.py:158-171, 336-352)."""
        B, S, d, K = self.B, self.S, self.d, self.K
        g = ops.gemm_conv
        rows = B * K
        cur = 0
        # the deformable cross-attention's value projections of every layer, in one pass over
        # the memory
        g(self.mem.view(B * S, d), *self.w_value, out=self.value.view(B * S, -1))
        for i, w in enumerate(self.w_layers):
            tgt = self.tgt32[cur]
            # query position of the current boxes
            g(self.qin.view(rows, 64), *self.w_qpos[0], act="relu", out=self.qp1.view(rows, -1))
            g(self.qp1.view(rows, -1), *self.w_qpos[1], out=self.pos.view(rows, d))
            # self-attention: q = k = tgt + pos, v = tgt
            ops.add_rows(tgt, self.pos, self.q16)
            g(self.q16.view(rows, d), *w["qk"], out=self.qk.view(rows, 2 * d))
            g(self.tgt16.view(rows, d), *w["v"], out=self.vv.view(rows, d))
            ops.attention(self.qk[..., :d], self.qk[..., d:], self.vv, self.heads, out=self.att_q)
            g(self.att_q.view(rows, d), *w["o"], out=self.sa_q.view(rows, d))
            n1, n2, n3 = w["n"]
            # the layer input tgt stays intact: the corner head of the next layer reads it
            ops.layernorm(tgt, n1[0], n1[1], n1[2], b=self.sa_q, y32=self.mid32, pos=self.pos, yp16=self.qc16)
            # deformable cross-attention on the memory
            g(self.qc16.view(rows, d), *w["offatt"], out=self.offatt.view(rows, -1))
            n_off = w["n_off"]
            ref = self.ref16 if i == 0 else self.box
            ops.deform_sample(self.value[..., i * d:(i + 1) * d], self.shapes, self.offatt[..., :n_off],
                              self.offatt[..., n_off:], ref, self.heads, self.points, out=self.samp)
            g(self.samp.view(rows, d), *w["cout"], out=self.cross.view(rows, d))
            ops.layernorm(self.mid32, n2[0], n2[1], n2[2], b=self.cross, y32=self.mid32, y16=self.ffn_in)
            g(self.ffn_in.view(rows, d), *w["f1"], act="relu", out=self.ffn_q.view(rows, -1))
            g(self.ffn_q.view(rows, -1), *w["f2"], out=self.ffn2_q.view(rows, d))
            nxt = self.tgt32[1 - cur]
            ops.layernorm(self.mid32, n3[0], n3[1], n3[2], b=self.ffn2_q, y32=nxt, y16=self.tgt16)
            # box heads
            if i == 0:
                self._mlp(self.w_pre, self.tgt16, [self.h1, self.h2], self.pb)
                head_in = self.tgt16
            else:
                ops.add_rows(nxt, tgt, self.head_in)  # tgt + tgt_detach of the previous layer
                head_in = self.head_in
            self._mlp(self.w_corner[i], head_in, [self.h1, self.h2], self.head)
            ops.box_dec(i == 0, self.head, self.corners, self.project, self.reg_scale, self.ref_init, self.box,
                        prebox=self.pb, ref16=self.ref16, qin=self.qin)
            cur = 1 - cur
        self.cur = cur
        tgt = self.tgt32[cur]
        g(self.tgt16.view(rows, d), *self.w_cls[-1], out=self.logits.view(rows, self.nc))
        self._mlp(self.w_id, self.tgt16, [self.idh], self.idv)
        ops.l2norm_rows(self.idv.view(rows, -1), self.id_embed.view(rows, -1))

    # ------------------------------------------------------------ public
    @torch.no_grad()
    def run(self, p8):
        """p8: [B, C8, h8, w8] (NCHW view of an NHWC map, as the engine's outputs_nchw gives,
        or any layout; fp16 or fp32) -> output dict (views of this object's buffers)."""
        want = (self.B, self.c8, *self.shapes[0])
        if tuple(p8.shape) != want or not p8.is_cuda:
            raise ValueError(f"p8: expected a CUDA tensor of shape {want}, got {tuple(p8.shape)}")
        x = p8.permute(0, 2, 3, 1)
        if x.dtype != torch.float16 or not x.is_contiguous():
            x = x.contiguous().half()
        self._x8in = x
        self.core(x)
        self.encoder()
        self.decoder()
        return self.outputs()

    def outputs(self):
        tgt = self.tgt32[getattr(self, "cur", 0)]
        return {"pred_logits": self.logits, "pred_boxes": self.box, "pred_corners": self.corners,
                "ref_init": self.ref_init, "enc_logits": self.enc_logits_sel, "enc_boxes": self.ref16,
                "embed": tgt, "boxes": self.box, "id_embed": self.id_embed, "n_track": 0,
                "memory": self.mem, "top": self.top}

    def capture(self, p8):
        """Capture run(p8) as one CUDA graph; replay() then reruns it on p8's storage."""
        self.run(p8)  # outside capture: first-call setup of the kernels
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.run(p8)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run(p8)
        self._graph_in = p8
        return self.outputs()

    def replay(self):
        self.graph.replay()
        return self.outputs()

    def __call__(self, p8):
        if self.graph is not None and p8 is self._graph_in:
            return self.replay()
        return self.run(p8)


def install(video):
    """Run a reference ``SarbonVideo``'s detector on B200Detector.

    ``SarbonVideo._detect`` (sarbon/inference/video.py:120-137) calls ``self._run_det(p8)``,
    which runs ``self.det(None, p8=p8)`` under autocast, and captures it as a CUDA graph.
    This replaces ``_run_det`` on the instance: the first call builds a B200Detector over
    ``video.det``'s weights for p8's shape (outside the graph capture: ``_detect`` warms up
    first), and every call launches its kernels on the current stream, so the video's own
    graph captures and replays them.  Returns the video."""
    state = {}

    def run_det(p8):
        d = state.get("det")
        if d is None or (d.B, *d.shapes[0]) != (p8.shape[0], p8.shape[2], p8.shape[3]):
            d = state["det"] = B200Detector(video.det, p8.shape[0], p8.shape[2], p8.shape[3], device=p8.device)
        return d.run(p8)

    video._run_det = run_det
    video.b200_detector = state
    return video
