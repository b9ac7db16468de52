"""The Laya DecisionModel (ModernBERT encoder + type embedding + two PyTorch
pre-norm encoder layers + marker scorer + action head) on any backend of the
contract — the host-side mirror of packages/laya/src/model.ts:

- ``DecisionModel.headLayer``    model.ts:124-137
- ``DecisionModel.uploadBatch``  model.ts:146-170
- ``DecisionModel.forwardCore``  model.ts:182-235
- ``DecisionModel.compiled``     model.ts:250-272 (Backend.compile = CUDA graphs)
- ``DecisionModel.readOutputs``  model.ts:275-285
- ``loadDecisionModel``          model.ts:319-366 (+ buildHeadWeights :368-405)

Every op goes through the backend, so on ``createCudaBackend()`` the whole
``predict()`` forward runs on the GPU.
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np

from . import compose as Cm
from .host import HostTensor, to_f32
from .modernbert import ModernBert, attentionMasks, disposeWeight, loadModernBert, parseModernBertConfig, uploadAs

HEAD_EPS = 1e-5  # PyTorch nn.LayerNorm / MLX nn.LayerNorm default (model.ts:30)


class DecisionModel:
    def __init__(self, backend, encoder: ModernBert, weights: dict, dtype: str, nAct: int):
        self.backend = backend
        self.encoder = encoder
        self.weights = weights
        self.dtype = dtype
        self.nAct = nAct
        self.hiddenSize = encoder.config["hiddenSize"]
        self.headHeads = max(1, self.hiddenSize // 64)

    def headLayer(self, j: int, x, mask):
        """model.ts:124-137: PyTorch pre-norm TransformerEncoderLayer (ReLU FFN), mask bool [B,1,1,L]."""
        b, w = self.backend, self.weights["head"][j]

        def f():
            B, L, D = x.shape
            nh = self.headHeads
            hd = D // nh
            h = b.layerNorm(x, w["norm1.weight"], w["norm1.bias"], HEAD_EPS)
            qkv = b.transpose(b.reshape(Cm.linearAny(b, h, w["inProj"], w["inProjBias"]), [B, L, 3, nh, hd]), [2, 0, 3, 1, 4])
            q, k, v = [b.reshape(t, [B, nh, L, hd]) for t in b.split(qkv, 3, 0)]
            att = b.reshape(b.transpose(b.sdpa(q, k, v, mask, hd ** -0.5), [0, 2, 1, 3]), [B, L, D])
            x1 = b.add(x, Cm.linearAny(b, att, w["outProj"], w["outProjBias"]))
            ff = Cm.linearAny(b, b.relu(Cm.linearAny(b, b.layerNorm(x1, w["norm2.weight"], w["norm2.bias"], HEAD_EPS),
                                                     w["linear1"], w["linear1Bias"])), w["linear2"], w["linear2Bias"])
            return b.add(x1, ff)
        return b.scope(f)

    def uploadBatch(self, batch: dict) -> dict:
        """model.ts:146-170. batch: inputIds i32 [B*L], attentionMask u8 [B*L], size, length,
        markerCount, markerPos i32 [B*M], markerMask u8 [B*M], qtype i32 [B]."""
        b = self.backend
        B, L, M = batch["size"], batch["length"], batch["markerCount"]
        if M < 2:
            raise ValueError("DecisionModel: markerCount must be >= 2 (collate pads to two slots)")
        full, sliding = attentionMasks(batch["attentionMask"], B, L, self.encoder.config["localAttention"])
        pos = np.maximum(np.asarray(batch["markerPos"], np.int32).reshape(B, M), 0)
        mm = np.asarray(batch["markerMask"], np.uint8).reshape(B, M)
        k = np.maximum(mm.astype(np.int64).sum(axis=1), 2).astype(np.float32)
        made = {}
        try:
            made["inputIds"] = b.fromHost(HostTensor("i32", (B, L), np.asarray(batch["inputIds"], np.int32).reshape(B, L)))
            made["fullMask"] = b.fromHost(full)
            made["slidingMask"] = b.fromHost(sliding)
            made["headMask"] = b.fromHost(HostTensor("bool", (B, 1, 1, L), np.asarray(batch["attentionMask"], np.uint8).reshape(B, 1, 1, L)))
            made["qtype"] = b.fromHost(HostTensor("i32", (B,), np.asarray(batch["qtype"], np.int32)))
            made["markerPos"] = b.fromHost(HostTensor("i32", (B, M), pos))
            made["markerMask"] = b.fromHost(HostTensor("bool", (B, M), mm))
            made["k"] = b.fromHost(HostTensor("f32", (B,), k))
        except BaseException:
            for t in made.values():
                b.dispose(t)
            raise
        return made

    def disposeInputs(self, inp: dict) -> None:
        for t in inp.values():
            self.backend.dispose(t)

    def forwardCore(self, inp: dict, onStage: Optional[Callable] = None) -> dict:
        """model.ts:182-235 → {"logits": f32 [B, M] (masked slots −1e4), "act": f32 [B, nAct]}."""
        b, w, enc = self.backend, self.weights, self.encoder
        B, L = inp["inputIds"].shape
        M = inp["markerPos"].shape[1]
        D = self.hiddenSize
        kept = []

        def emit(name, t):
            own = onStage is not None and onStage(name, t) is True
            if own:
                kept.append(t)
            return own

        cst = w["constants"]

        def f():
            masks = {"full_attention": inp["fullMask"], "sliding_attention": inp["slidingMask"]}
            x = enc.embeddings(inp["inputIds"])
            owned = emit("embeddings", x)
            for i in range(enc.config["numHiddenLayers"]):
                nxt = enc.layer(i, x, masks[enc.config["layerTypes"][i]])
                if not owned:
                    b.dispose(x)
                x = nxt
                owned = emit(f"encoder.layers.{i}", x)
            encOut = enc.finalNorm(x)
            if not owned:
                b.dispose(x)
            emit("encoder.final_norm", encOut)
            h = b.add(encOut, b.reshape(Cm.embeddingAny(b, w["typeEmb"], inp["qtype"]), [B, 1, D]))
            emit("type_emb_added", h)
            for j in range(len(w["head"])):
                h = self.headLayer(j, h, inp["headMask"])
                emit(f"head.layers.{j}", h)
            markers = b.gatherRows(h, inp["markerPos"])
            s = w["scorer"]
            scored = Cm.linearAny(b, b.gelu(Cm.linearAny(b, b.layerNorm(markers, s["norm.weight"], s["norm.bias"], HEAD_EPS),
                                                         s["w1"], s["b1"])), s["w2"], s["b2"])
            logits = b.where(inp["markerMask"], b.cast(b.reshape(scored, [B, M]), "f32"), cst["maskedLogit"])
            p = b.softmax(logits, -1)
            plogp = b.mul(p, b.log(b.maximum(p, cst["probFloor"])))
            entropy = b.div(b.scale(b.sum(plogp, -1), -1), b.log(inp["k"]))
            top = b.slice(b.sort(p, -1), [0, M - 2], [B, M])
            top2 = b.slice(top, [0, 0], [B, 1])
            top1 = b.slice(top, [0, 1], [B, 2])
            kScaled = b.div(b.reshape(inp["k"], [B, 1]), cst["kScale"])
            features = b.concat([top1, b.sub(top1, top2), b.reshape(entropy, [B, 1]), kScaled], -1)
            cls = b.cast(b.reshape(b.slice(h, [0, 0, 0], [B, 1, D]), [B, D]), "f32")
            pooled = b.cast(b.concat([cls, features], -1), self.dtype)
            a = w["act"]
            act = b.cast(Cm.linearAny(b, b.gelu(Cm.linearAny(b, pooled, a["w1"], a["b1"])), a["w2"], a["b2"]), "f32")
            return [logits, act, *kept]
        out = b.scope(f)
        return {"logits": out[0], "act": out[1]}

    def forwardTensors(self, batch: dict, onStage: Optional[Callable] = None) -> dict:
        inp = self.uploadBatch(batch)
        try:
            return self.forwardCore(inp, onStage)
        finally:
            self.disposeInputs(inp)

    def compiled(self) -> Optional[Callable[[dict], dict]]:
        """model.ts:250-272: a ``forwardTensors`` equivalent through
        ``backend.compile`` (here one CUDA graph per input shape signature),
        or None when the backend has no ``compile``. No stage observation."""
        b = self.backend
        if not hasattr(b, "compile"):
            return None
        names = ("inputIds", "fullMask", "slidingMask", "headMask", "qtype", "markerPos", "markerMask", "k")

        def core(*ts):
            r = self.forwardCore(dict(zip(names, ts)))
            return [r["logits"], r["act"]]
        fn = b.compile(core)

        def run(batch: dict) -> dict:
            inp = self.uploadBatch(batch)
            try:
                logits, act = fn(*[inp[n] for n in names])
                return {"logits": logits, "act": act}
            finally:
                self.disposeInputs(inp)
        return run

    def readOutputs(self, r: dict) -> dict:
        """model.ts:275-285: flush, read both (f32), free."""
        b = self.backend
        try:
            b.flush(r["logits"], r["act"])
            return {"logits": to_f32(b.read(r["logits"])), "act": to_f32(b.read(r["act"])), "nAct": self.nAct}
        finally:
            b.dispose(r["logits"])
            b.dispose(r["act"])

    def forward(self, batch: dict, onStage: Optional[Callable] = None) -> dict:
        return self.readOutputs(self.forwardTensors(batch, onStage))

    def dispose(self) -> None:
        self.encoder.dispose()
        b, w = self.backend, self.weights
        for l in w["head"]:
            for t in l.values():
                disposeWeight(b, t)
        for t in (w["typeEmb"], *w["scorer"].values(), *w["act"].values(), *w["constants"].values()):
            disposeWeight(b, t)


def loadDecisionModel(b, encoderConfig: dict, agentConfig: dict, get: Callable[[str], object], dtype: str = "f32") -> DecisionModel:
    """model.ts:319-366 / buildHeadWeights :368-405 (laya-mlx names; PyTorch spellings accepted)."""
    config = encoderConfig if "hiddenSize" in encoderConfig else parseModernBertConfig(encoderConfig)
    D = config["hiddenSize"]
    head_layers = agentConfig.get("head_layers", 2)
    nAct = len(agentConfig.get("act_costs") or {}) + 1
    made = []

    def need(names, shape, matrix=False):
        for n in names:
            h = get(n)
            if h is None:
                continue
            if tuple(h.shape) != tuple(shape):
                raise ValueError(f"DecisionModel: {n} has shape {list(h.shape)}, want {list(shape)}")
            t = uploadAs(b, h, dtype)
            made.append(t)
            return t
        raise KeyError(f"DecisionModel: missing weight {names[0]}")

    seq = lambda p, i, what: [f"{p}.layers.{i}.{what}", f"{p}.{i}.{what}"]
    encoder = loadModernBert(b, config, get, dtype, prefix="encoder.")
    try:
        head = []
        for j in range(head_layers):
            p = f"head.layers.{j}"
            head.append({
                "norm1.weight": need([f"{p}.norm1.weight"], [D]), "norm1.bias": need([f"{p}.norm1.bias"], [D]),
                "norm2.weight": need([f"{p}.norm2.weight"], [D]), "norm2.bias": need([f"{p}.norm2.bias"], [D]),
                "inProj": need([f"{p}.self_attn.in_proj.weight", f"{p}.self_attn.in_proj_weight"], [3 * D, D], True),
                "inProjBias": need([f"{p}.self_attn.in_proj.bias", f"{p}.self_attn.in_proj_bias"], [3 * D]),
                "outProj": need([f"{p}.self_attn.out_proj.weight"], [D, D], True),
                "outProjBias": need([f"{p}.self_attn.out_proj.bias"], [D]),
                "linear1": need([f"{p}.linear1.weight"], [4 * D, D], True), "linear1Bias": need([f"{p}.linear1.bias"], [4 * D]),
                "linear2": need([f"{p}.linear2.weight"], [D, 4 * D], True), "linear2Bias": need([f"{p}.linear2.bias"], [D]),
            })
        weights = {
            "head": head,
            "typeEmb": need(["type_emb.weight"], [3, D], True),
            "scorer": {"norm.weight": need(seq("scorer", 0, "weight"), [D]), "norm.bias": need(seq("scorer", 0, "bias"), [D]),
                       "w1": need(seq("scorer", 1, "weight"), [D, D], True), "b1": need(seq("scorer", 1, "bias"), [D]),
                       "w2": need(seq("scorer", 3, "weight"), [1, D], True), "b2": need(seq("scorer", 3, "bias"), [1])},
            "act": {"w1": need(seq("act_head", 0, "weight"), [256, D + 4], True), "b1": need(seq("act_head", 0, "bias"), [256]),
                    "w2": need(seq("act_head", 2, "weight"), [nAct, 256], True), "b2": need(seq("act_head", 2, "bias"), [nAct])},
            # f32 whatever the model dtype (model.ts:342-347)
            "constants": {k: b.fromHost(HostTensor("f32", (1,), np.array([v], np.float32)))
                          for k, v in (("maskedLogit", -1e4), ("probFloor", 1e-9), ("kScale", 255.0))},
        }
    except BaseException:
        for t in made:
            disposeWeight(b, t)
        encoder.dispose()
        raise
    return DecisionModel(b, encoder, weights, dtype, nAct)
