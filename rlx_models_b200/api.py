"""High-level API: ``load(model)`` -> :class:`LLM` with generate / stream / logits.

The B200 counterpart of the reference's runner builders and `auto_runner`
(rlx-qwen3 src/high_level_runner.rs:90-181 `Qwen3Runner::builder()...build()`,
:515-970 `generate` / `predict_logits` / `cache_prefix`; rlx-models
src/run.rs:76-175 `auto_runner`, which sniffs the architecture from the
checkpoint). ``model`` may be

* a local directory with ``config.json`` + safetensors (HF layout, same tensor
  names as the reference's loaders),
* an HF repo id resolved offline from the local HF cache (``org/name``), or
* a named shape (``qwen3-0.6b``, ``qwen3-8b``, ``gpt-oss-120b`` ...) with seeded
  random weights, which is what the benchmarks use.
"""
from __future__ import annotations

import os
from typing import Iterator

import torch

from . import config as C
from .registry import build_model
from .runtime.engine import EngineConfig, LLMEngine, RequestOutput, SamplingParams
from .weights.weight_map import WeightMap


def parse_model_ref(ref: str) -> tuple[str, str | None, str | None]:
    """``org/name[:QUANT][@rev]`` -> (org/name, quant, rev); local paths pass through.

    The hub reference syntax of the reference's model hub (rlx-model-hub):
    QUANT names a quantised variant (e.g. ``mxfp4``, ``fp8``), ``rev`` a
    snapshot revision in the cache."""
    if os.path.exists(ref):
        return ref, None, None
    name, _, rev = ref.partition("@")
    name, _, quant = name.partition(":")
    return name, (quant or None), (rev or None)


GGUF_QUANT_PREFERENCE = ("Q4_K_M", "Q4_K_S", "Q5_K_M", "Q6_K", "Q8_0", "Q4_0", "F16", "BF16")


def pick_gguf(directory: str, quant: str | None = None) -> str | None:
    """The GGUF file of ``directory`` whose name carries ``quant`` (case
    insensitive), else the first match in the default quant preference order
    (the hub's "QUANT" selection rule), else the only GGUF file."""
    files = sorted(f for f in os.listdir(directory) if f.lower().endswith(".gguf"))
    if not files:
        return None
    for q in ((quant,) if quant else ()) + GGUF_QUANT_PREFERENCE:
        for f in files:
            if q.lower() in f.lower():
                return os.path.join(directory, f)
    if quant:
        raise FileNotFoundError(f"no GGUF file for quant {quant!r} in {directory}: {files}")
    return os.path.join(directory, files[0])


def resolve_model_path(model: str) -> str | None:
    """Local dir or .gguf file, or an HF id found in the offline HF cache
    (snapshots/<rev>)."""
    if os.path.isdir(model) or (os.path.isfile(model) and model.lower().endswith(".gguf")):
        return model
    if os.path.isfile(model) and model.lower().endswith(".rlxp"):  # packed model: unpack once into the cache
        from .weights.assets import materialize
        return materialize(model)
    if model.startswith("ollama:") or model.startswith("local:"):  # discovery queries (weights/discover.py)
        from .weights.discover import resolve
        return resolve(model.split(":", 1)[1] if model.startswith("local:") else model)
    if "/" in model:
        name, _, rev = parse_model_ref(model)
        root = os.environ.get("HF_HUB_CACHE") or os.path.join(
            os.environ.get("HF_HOME", os.path.expanduser("~/.cache/huggingface")), "hub")
        d = os.path.join(root, "models--" + name.replace("/", "--"), "snapshots")
        if os.path.isdir(d):
            snaps = sorted(os.listdir(d))
            if rev and rev in snaps:
                return os.path.join(d, rev)
            if snaps:
                return os.path.join(d, snaps[-1])
    from . import config as _C
    if not any(model == k or model.startswith(k) for k in _C.PRESETS):
        # not a named random-init shape: look in other tools' caches (LM Studio, Ollama, HF, ...)
        from .weights.discover import resolve
        return resolve(model)
    return None


class LLM:
    """A loaded language model plus its serving engine (one process, TP rank)."""

    def __init__(self, model, engine_config: EngineConfig | None = None, tokenizer=None):
        self.model = model
        self.engine = LLMEngine(model, engine_config)
        self.tokenizer = tokenizer

    @property
    def config(self):
        return self.model.cfg

    def _encode(self, p):
        if isinstance(p, str):
            if self.tokenizer is None:
                raise ValueError("string prompts need a tokenizer")
            return self.tokenizer.encode(p)
        return list(p)

    def generate(self, prompts, params: SamplingParams | list[SamplingParams] | None = None) -> list[RequestOutput]:
        single = isinstance(prompts, str) or (prompts and isinstance(prompts[0], int))
        plist = [prompts] if single else list(prompts)
        outs = self.engine.generate([self._encode(p) for p in plist], params)
        return outs[:1] if single else outs

    def stream(self, prompt, params: SamplingParams | None = None) -> Iterator[int]:
        """Yield tokens of one request as they are produced."""
        sid = self.engine.add_request(self._encode(prompt), params)
        seen = 0
        while True:
            done = {o.seq_id: o for o in self.engine.step()}
            st = self.engine.requests.get(sid)
            toks = done[sid].token_ids if sid in done else (st.tokens if st else [])
            for t in toks[seen:]:
                yield t
            seen = len(toks)
            if sid in done or not self.engine.has_unfinished():
                return

    @torch.no_grad()
    def embed(self, prompts, pooling: str = "last", normalize: bool = True) -> torch.Tensor:
        """Sequence embeddings [N, H] (fp32) from the final-normed hidden states
        of one batched prefill: ``pooling`` "last" (the last token, as
        decoder embedding models such as Qwen3-Embedding use), "mean" or
        "first"; L2-normalised unless ``normalize`` is False."""
        from .models.decoder import ForwardBatch
        single = isinstance(prompts, str) or (prompts and isinstance(prompts[0], int))
        seqs = [self._encode(p) for p in ([prompts] if single else prompts)]
        dev = self.model.device
        nbs = [(len(s) + 15) // 16 for s in seqs]
        W = max(nbs)
        tables = torch.zeros(len(seqs), W, dtype=torch.int32)
        slots, off = [], 0
        for i, (s, nb) in enumerate(zip(seqs, nbs)):
            tables[i, :nb] = torch.arange(off, off + nb, dtype=torch.int32)
            slots.append(torch.arange(off * 16, off * 16 + len(s), dtype=torch.int64))
            off += nb
        lens = [len(s) for s in seqs]
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
        kv = self.model.make_kv_cache(off)
        fb = ForwardBatch(input_ids=torch.tensor([t for s in seqs for t in s], dtype=torch.int32, device=dev),
                          positions=torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]).to(dev),
                          slots=torch.cat(slots).to(dev), num_decode=0, pre_block_tables=tables.to(dev),
                          pre_ctx_lens=torch.tensor(lens, dtype=torch.int32, device=dev), pre_cu_q=cu.to(dev),
                          pre_max_q=max(lens))
        h = self.model.forward_hidden(fb, kv).float()
        rows = []
        for i in range(len(seqs)):
            seg = h[int(cu[i]):int(cu[i + 1])]
            rows.append(seg[-1] if pooling == "last" else seg.mean(0) if pooling == "mean" else seg[0])
        e = torch.stack(rows)
        return torch.nn.functional.normalize(e, dim=-1) if normalize else e

    def logits(self, prompt) -> torch.Tensor:
        """fp32 next-token logits for every prompt position (prefill only)."""
        from .models.decoder import ForwardBatch
        ids = self._encode(prompt)
        T = len(ids)
        dev = self.model.device
        kv = self.model.make_kv_cache((T + 15) // 16)
        nb = (T + 15) // 16
        fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32, device=dev),
                          positions=torch.arange(T, dtype=torch.int32, device=dev),
                          slots=torch.arange(T, dtype=torch.int64, device=dev), num_decode=0,
                          pre_block_tables=torch.arange(nb, dtype=torch.int32, device=dev).view(1, -1),
                          pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                          pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), pre_max_q=T)
        return self.model.forward(fb, kv)


def load(model: str, *, device: str | torch.device = "cuda", tp_rank: int = 0, tp_size: int = 1, comm=None,
         seed: int = 0, engine_config: EngineConfig | None = None, config: C.DecoderConfig | None = None) -> LLM:
    """Load a model by path, HF id (offline cache) or named shape (random init)."""
    path = resolve_model_path(model)
    tok = None
    gguf_file = None
    if path is not None:
        if os.path.isfile(path):
            gguf_file = path
        elif not os.path.exists(os.path.join(path, "config.json")):
            gguf_file = pick_gguf(path, parse_model_ref(model)[1])
    if gguf_file is not None:
        from .weights.gguf import GGUFWeights
        weights = GGUFWeights(gguf_file, device=device)  # quantised blocks expand on the GPU
        cfg = config or weights.config
    elif path is not None:
        from .models.deepseek import DeepseekConfig, is_deepseek_config
        from .models.qwen35 import Qwen35Config, is_qwen35_config
        if config is None and is_deepseek_config(path):  # MLA + DeepSeekMoE family
            config = DeepseekConfig.from_file(path)
        elif config is None and is_qwen35_config(path):  # Gated DeltaNet hybrid
            config = Qwen35Config.from_file(path)
        else:
            from .models.lfm2 import Lfm2Config, is_lfm2_config
            from .models.mamba2 import SSMConfig, is_ssm_config
            from .models.minimax import MiniMaxConfig, is_minimax_config
            if config is None and is_lfm2_config(path):  # short-conv hybrid
                config = Lfm2Config.from_file(path)
            elif config is None and is_minimax_config(path):  # lightning-attention hybrid
                config = MiniMaxConfig.from_file(path)
            elif config is None and is_ssm_config(path):  # Mamba-2 (SSD) and its attention hybrids
                config = SSMConfig.from_file(path)
            else:
                from .models.mamba1 import Mamba1Config, is_mamba1_config
                if config is None and is_mamba1_config(path):  # Mamba-1 selective scan, Jamba
                    config = Mamba1Config.from_file(path)
        cfg = config or C.DecoderConfig.from_file(path)
        from .weights.mlx import MLXWeights
        if MLXWeights.is_mlx_dir(path):  # MLX affine group-quantised checkpoint
            weights = MLXWeights(path, device=device)
        else:
            weights = WeightMap.from_dir(path)
            from .weights.aliases import LanguageModelView
            if getattr(cfg, "model_type", "") != "llama4_text" and LanguageModelView.applies(weights):
                weights = LanguageModelView(weights)  # the text model of a multimodal checkpoint
        try:
            from .tokenizer import load_tokenizer
            tok = load_tokenizer(path)
        except Exception:
            tok = None
    else:
        cfg = config or C.preset(model)
        weights = None  # random init on the device, per rank
    m = build_model(cfg, weights, device=device, tp_rank=tp_rank, tp_size=tp_size, comm=comm, seed=seed)
    return LLM(m, engine_config, tok)


def load_transcriber(model: str, *, device: str | torch.device = "cuda", language: str | None = "en",
                     task: str = "transcribe"):
    """Whisper, Moonshine, Parakeet-CTC or wav2vec 2.0 CTC checkpoint (local dir / offline HF id)
    -> object with ``transcribe(audio, sample_rate)``."""
    import json
    from .models.whisper import SpeechToText, WhisperConfig, WhisperModel
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local speech checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    tok = None
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json", "vocab.json")):
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    if raw.get("model_type") == "moonshine":
        from .models.moonshine import MoonshineConfig, MoonshineModel, MoonshineTranscriber
        return MoonshineTranscriber(MoonshineModel(MoonshineConfig.from_dict(raw), WeightMap.from_dir(path),
                                                   device=device), tok)
    if raw.get("model_type") in ("wav2vec2", "wav2vec2-ctc"):
        from .models.wav2vec2 import Wav2Vec2Config, Wav2Vec2CTC, Wav2Vec2Transcriber
        return Wav2Vec2Transcriber(Wav2Vec2CTC(Wav2Vec2Config.from_dict(raw), WeightMap.from_dir(path), device=device),
                                   tok, normalize=raw.get("do_normalize", True))
    if raw.get("model_type") == "wav2vec2-bert":
        from .models.w2v_bert import W2vBertConfig, W2vBertCTC, W2vBertTranscriber
        return W2vBertTranscriber(W2vBertCTC(W2vBertConfig.from_dict(raw), WeightMap.from_dir(path), device=device), tok)
    if raw.get("model_type") == "parakeet_ctc":
        from .models.parakeet import ParakeetConfig, ParakeetCTC, ParakeetTranscriber
        return ParakeetTranscriber(ParakeetCTC(ParakeetConfig.from_dict(raw), WeightMap.from_dir(path), device=device),
                                   tok)
    cfg = WhisperConfig.from_dict(raw)
    return SpeechToText(WhisperModel(cfg, WeightMap.from_dir(path), device=device), tok, language, task)


def load_codec(model: str, *, device: str | torch.device = "cuda"):
    """Neural audio codec checkpoint (local dir / offline HF id): DAC (transformers'
    or the original Descript layout; ``encode(pcm) -> codes``, ``decode(codes)
    -> pcm``, ``roundtrip``) or EnCodec (``encode(pcm, bandwidth) -> (codes,
    scales, pad)``, ``decode(codes, scales, pad)``, the transformers layout) or Mimi
    (``encode(pcm, num_quantizers) -> codes``, ``decode(codes)``)."""
    import json
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local codec checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    if raw.get("model_type", "dac") == "dac":
        from .models.dac import DacConfig, DacModel
        return DacModel(DacConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    if raw.get("model_type") == "mimi":
        from .models.mimi import MimiConfig, MimiModel
        return MimiModel(MimiConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    if raw.get("model_type") == "encodec":
        from .models.encodec import EncodecConfig, EncodecModel
        return EncodecModel(EncodecConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    raise NotImplementedError(f"codec model_type {raw.get('model_type')!r}")


class Segmenter:
    """Segment Anything: an image and point / box prompts (in the image's own
    pixel coordinates) -> boolean masks at the image's size and IoU scores.
    ``set_image`` keeps the encoder output for further prompts on the same image."""

    MEAN, STD = (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)

    def __init__(self, model):
        self.model = model
        self.size = model.cfg.vision.image_size
        self._emb = None
        self._sizes = None

    def preprocess(self, image):
        """Longest edge to the model's input size (bilinear), ImageNet
        normalisation, zero padding to a square at the bottom / right."""
        from PIL import Image

        from .utils.preprocess import load_image, normalize, to_tensor
        img = load_image(image)
        w, h = img.size
        s = self.size / max(h, w)
        nh, nw = int(h * s + 0.5), int(w * s + 0.5)
        t = normalize(to_tensor(img.resize((nw, nh), resample=Image.BILINEAR)), self.MEAN, self.STD)
        t = torch.nn.functional.pad(t, (0, self.size - nw, 0, self.size - nh))
        return t[None], (h, w), (nh, nw)

    def set_image(self, image) -> None:
        px, orig, resized = self.preprocess(image)
        self._emb = self.model.image_embeddings(px)
        self._sizes = (orig, resized)

    def segment(self, image=None, points=None, labels=None, boxes=None, multimask: bool = True):
        """points [P, n, 2] (x, y) with labels [P, n] (1 foreground, 0
        background), and / or boxes [P, 4] (x0, y0, x1, y1) -> (masks [P, k, H, W]
        bool, iou [P, k]); k = 3 with ``multimask`` else 1."""
        from .models.sam import upscale_masks
        if image is not None:
            self.set_image(image)
        if self._emb is None:
            raise ValueError("no image: pass one or call set_image first")
        (h, w), (nh, nw) = self._sizes
        scale = torch.tensor([nw / w, nh / h])
        pts = None if points is None else (torch.as_tensor(points, dtype=torch.float32) * scale)[None]
        lab = None if labels is None else torch.as_tensor(labels)[None]
        bx = None if boxes is None else (torch.as_tensor(boxes, dtype=torch.float32).view(-1, 2, 2) * scale).view(1, -1, 4)
        masks, iou = self.model.segment(points=pts, labels=lab, boxes=bx, image_embeddings=self._emb,
                                        multimask=multimask)
        return upscale_masks(masks[0].cpu(), (h, w), (nh, nw), self.size), iou[0].cpu()


def load_segmenter(model: str, *, device: str | torch.device = "cuda") -> Segmenter:
    """SAM checkpoint (transformers' SamModel layout; local dir / offline HF id) -> ``Segmenter``."""
    import json
    from .models.sam import SamConfig, SamModel
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local SAM checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    return Segmenter(SamModel(SamConfig.from_dict(raw), WeightMap.from_dir(path), device=device))


class Translator:
    """Many-to-many translation (NLLB-200 / M2M-100): ``translate(texts,
    src_lang, tgt_lang)`` with the checkpoint's tokenizer (language codes as
    the tokenizer names them, e.g. "eng_Latn" / "fra_Latn" for NLLB)."""

    def __init__(self, model, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer

    def translate(self, texts, src_lang: str, tgt_lang: str, max_new_tokens: int = 128) -> list:
        if self.tokenizer is None:
            raise ValueError("no tokenizer next to the checkpoint; use model.generate on token ids")
        single = isinstance(texts, str)
        texts = [texts] if single else list(texts)
        self.tokenizer.src_lang = src_lang
        enc = self.tokenizer(texts, return_tensors="pt", padding=True)
        ids = self.model.generate(enc["input_ids"], forced_bos=self.tokenizer.convert_tokens_to_ids(tgt_lang),
                                  max_new_tokens=max_new_tokens)
        out = [self.tokenizer.decode(x, skip_special_tokens=True) for x in ids]
        return out[0] if single else out


def load_translator(model: str, *, device: str | torch.device = "cuda") -> Translator:
    """NLLB / M2M-100 checkpoint (local dir / offline HF id) -> ``Translator``."""
    import json
    from .models.nllb import NllbConfig, NllbTranslator
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local translation checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    tok = None
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "sentencepiece.bpe.model",
                                                            "tokenizer_config.json")):
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    return Translator(NllbTranslator(NllbConfig.from_dict(raw), WeightMap.from_dir(path), device=device), tok)


def load_forecaster(model: str, *, device: str | torch.device = "cuda"):
    """TimesFM checkpoint (transformers' TimesFmModelForPrediction layout; local
    dir / offline HF id) -> model with ``forecast(series, freq, horizon, ...)``."""
    import json
    from .models.timesfm import TimesFm, TimesFmConfig
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local forecasting checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    return TimesFm(TimesFmConfig.from_dict(raw), WeightMap.from_dir(path), device=device)


class SpeechGenerator:
    """Text to speech with CSM: ``speak(text, speaker=0)`` formats the prompt
    as the checkpoint's processor does ("[speaker]text"), generates Mimi frames
    greedily and decodes them to 24 kHz audio."""

    def __init__(self, model, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer

    def speak(self, text: str, speaker: int = 0, max_frames: int = 125) -> torch.Tensor:
        if self.tokenizer is None:
            raise ValueError("no tokenizer next to the checkpoint; use model.speak on token ids")
        ids = self.tokenizer(f"[{speaker}]{text}", return_tensors="pt")["input_ids"][0]
        return self.model.speak(ids, max_frames=max_frames)


def load_speech_generator(model: str, *, device: str | torch.device = "cuda") -> SpeechGenerator:
    """CSM checkpoint (transformers' CsmForConditionalGeneration layout, Mimi codec
    included; local dir / offline HF id) -> ``SpeechGenerator``."""
    import json
    from .models.csm import CsmConfig, CsmModel
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local speech-generation checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    tok = None
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    return SpeechGenerator(CsmModel(CsmConfig.from_dict(raw), WeightMap.from_dir(path), device=device), tok)


def load_video_model(model: str, *, device: str | torch.device = "cuda"):
    """V-JEPA 2 checkpoint (encoder alone or with the attentive-probe classifier;
    local dir / offline HF id) -> model with ``features(video)`` and, for
    classifiers, ``classify(video)`` (video [B, T, 3, H, W], preprocessed)."""
    import json
    from .models.vjepa2 import VJEPA2, VJEPA2Config
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local video checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    return VJEPA2(VJEPA2Config.from_dict(raw), WeightMap.from_dir(path), device=device)


class Embedder:
    """Sentence embeddings from an encoder checkpoint (BERT family)."""

    def __init__(self, encoder, tokenizer=None, pooling: str = "mean"):
        self.encoder, self.tokenizer, self.pooling = encoder, tokenizer, pooling

    def embed(self, texts, normalize: bool = True) -> torch.Tensor:
        if isinstance(texts, str):
            texts = [texts]
        if texts and isinstance(texts[0], str):
            if self.tokenizer is None:
                raise ValueError("string inputs need a tokenizer")
            enc = self.tokenizer(list(texts), padding=True, truncation=True, return_tensors="pt")
            ids, mask = enc["input_ids"], enc["attention_mask"]
        else:
            seqs = [list(t) for t in texts]
            L = max(len(s) for s in seqs)
            ids = torch.zeros(len(seqs), L, dtype=torch.long)
            mask = torch.zeros(len(seqs), L, dtype=torch.long)
            for i, s in enumerate(seqs):
                ids[i, :len(s)] = torch.tensor(s)
                mask[i, :len(s)] = 1
        return self.encoder.embed(ids, mask, pooling=self.pooling, normalize=normalize)


class DecoderEmbedder(Embedder):
    """Sentence embeddings from a decoder-shaped trunk run over whole texts
    (EuroBERT: bidirectional attention): final-normed hidden states pooled
    over each text's tokens ("mean", "cls" = first token, "last")."""

    def __init__(self, cfg, weights, device, tokenizer=None, pooling: str = "mean", dense=()):
        from .weights.aliases import ModelPrefixView
        self.cfg, self.device = cfg, torch.device(device)
        self.dense = list(dense)  # sentence-transformers Dense layers after pooling: (W, b or None)
        weights = ModelPrefixView(weights)
        if self.device.type == "cuda":
            import dataclasses
            from .models.decoder import DecoderLM
            # an encoder trunk has no LM head: point the (unused) head at the embedding table
            trunk_cfg = dataclasses.replace(cfg, tie_word_embeddings=True)
            self.trunk, self.oracle = DecoderLM(trunk_cfg, weights, device=self.device), None
        else:
            from .models.oracle import DecoderOracle
            self.trunk, self.oracle = None, DecoderOracle(cfg, {k: weights[k] for k in weights.keys()})
        super().__init__(self, tokenizer, pooling)

    def hidden(self, ids: list[int]) -> torch.Tensor:
        if self.oracle is not None:
            return self.oracle.forward_hidden(torch.tensor(ids))[0]
        if any(L.window and len(ids) > L.window for L in self.trunk.layers):
            # the prefill kernel's non-causal mode has no window
            raise NotImplementedError("bidirectional sliding-window layers on the GPU: texts up to the window only")
        from .models.decoder import ForwardBatch
        T, dev = len(ids), self.device
        nb = (T + 15) // 16
        fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32, device=dev),
                          positions=torch.arange(T, dtype=torch.int32, device=dev),
                          slots=torch.arange(T, dtype=torch.int64, device=dev), num_decode=0,
                          pre_block_tables=torch.arange(nb, dtype=torch.int32, device=dev).view(1, -1),
                          pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                          pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), pre_max_q=T)
        return self.trunk.forward_hidden(fb, self.trunk.make_kv_cache(nb)).float()

    def __call__(self, ids: torch.Tensor, attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        """[B, L] padded ids -> [B, L, H] fp32 hidden states (zeros on padding)."""
        B, L = ids.shape
        out = torch.zeros(B, L, self.cfg.hidden_size)
        for b in range(B):
            keep = attention_mask[b].bool() if attention_mask is not None else torch.ones(L, dtype=torch.bool)
            out[b, keep] = self.hidden(ids[b][keep].tolist()).cpu()
        return out

    def embed(self, ids, attention_mask=None, pooling: str | None = None, normalize: bool = True):
        if isinstance(ids, (list, str)):  # texts / token lists through the Embedder front end
            return Embedder.embed(self, ids, normalize)
        h = self(ids, attention_mask)
        m = attention_mask.float() if attention_mask is not None else torch.ones(h.shape[:2])
        pooling = pooling or self.pooling
        if pooling == "cls":
            e = h[:, 0]
        elif pooling == "last":  # the last non-padding token of each text
            last = (m * torch.arange(m.shape[1])[None].float()).argmax(1)
            e = h[torch.arange(h.shape[0]), last]
        else:
            e = (h * m[..., None]).sum(1) / m.sum(1, keepdim=True).clamp_min(1.0)
        for w, b in self.dense:
            e = e @ w.t() + (b if b is not None else 0.0)
        return torch.nn.functional.normalize(e, dim=-1) if normalize else e


def _sentence_transformer_head(path: str):
    """(pooling mode, [(W, b)]) from a sentence-transformers layout
    (modules.json, N_Pooling/config.json, N_Dense/{config.json, weights});
    ("mean", []) when the directory has none. Dense layers with an identity
    activation only."""
    import json
    mf = os.path.join(path, "modules.json")
    if not os.path.exists(mf):
        return "mean", []
    pooling, dense = "mean", []
    for mod in json.load(open(mf)):
        kind, sub = mod.get("type", ""), os.path.join(path, mod.get("path", ""))
        if kind.endswith("Pooling"):
            pc = json.load(open(os.path.join(sub, "config.json")))
            pooling = "cls" if pc.get("pooling_mode_cls_token") else (
                "last" if pc.get("pooling_mode_lasttoken") else "mean")
        elif kind.endswith("Dense"):
            dc = json.load(open(os.path.join(sub, "config.json")))
            act = dc.get("activation_function", "torch.nn.modules.linear.Identity")
            if not act.endswith("Identity"):
                raise NotImplementedError(f"Dense activation {act}")
            w = WeightMap.from_dir(sub)
            dense.append((w.take("linear.weight").float(),
                          w.take("linear.bias").float() if "linear.bias" in w else None))
    return pooling, dense


def load_embedder(model: str, *, device: str | torch.device = "cuda", pooling: str = "mean") -> Embedder:
    """BERT-family checkpoint (local dir / offline HF id) -> ``Embedder``."""
    import json
    from .models.bert import BertConfig, BertEncoder
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local encoder checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    tok = None
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "vocab.txt")):
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    if raw.get("model_type") == "eurobert" or raw.get("use_bidirectional_attention"):
        # bidirectional decoder trunks: EuroBERT, EmbeddingGemma (Gemma-3 + pooling + Dense head)
        st_pool, dense = _sentence_transformer_head(path)
        return DecoderEmbedder(C.DecoderConfig.from_hf_dict(raw), WeightMap.from_dir(path), device, tok,
                               st_pool if dense else pooling, dense)
    if raw.get("model_type") == "nomic_bert":
        from .models.bert import NomicBertConfig, NomicBertEncoder
        return Embedder(NomicBertEncoder(NomicBertConfig.from_dict(raw), WeightMap.from_dir(path), device=device),
                        tok, pooling)
    return Embedder(BertEncoder(BertConfig.from_dict(raw), WeightMap.from_dir(path), device=device), tok, pooling)


class ImageEmbedder:
    """Image embeddings from a CLIP / SigLIP vision tower."""

    def __init__(self, encoder):
        self.encoder = encoder

    def pixels(self, images) -> torch.Tensor:
        from .utils import preprocess as P
        c = self.encoder.cfg
        if not hasattr(c, "family"):  # DINOv2: shortest edge 256, centre crop 224, ImageNet statistics
            return torch.stack([P.preprocess_image(im, size=256, crop=224, mean=P.IMAGENET_MEAN, std=P.IMAGENET_STD)
                                for im in images])
        if c.family == "siglip":
            return torch.stack([P.preprocess_image(im, size=(c.image_size, c.image_size), crop=None, mean=P.HALF,
                                                   std=P.HALF) for im in images])
        return torch.stack([P.preprocess_image(im, size=c.image_size, crop=c.image_size) for im in images])

    def embed(self, images, normalize: bool = True) -> torch.Tensor:
        """Paths, PIL images or HWC uint8 arrays -> [N, D] fp32 embeddings."""
        if not isinstance(images, (list, tuple)):
            images = [images]
        if hasattr(self.encoder, "embed_images"):  # SigLIP 2: NaFlex patches at each image's aspect ratio
            return self.encoder.embed_images(list(images), normalize=normalize)
        return self.encoder.embed(self.pixels(images), normalize=normalize)


def load_image_embedder(model: str, *, device: str | torch.device = "cuda") -> ImageEmbedder:
    """CLIP / SigLIP checkpoint (vision model alone or the full dual encoder) or
    a DINOv2 (with or without registers) / DINOv3 backbone (local dir / offline
    HF id) -> ``ImageEmbedder``."""
    import json
    from .models.vit import Dinov2Config, Dinov2Encoder, Dinov3Config, Dinov3Encoder, VisionConfig, VisionEncoder
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local vision checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    if raw.get("model_type") in ("dinov2", "dinov2_with_registers"):
        return ImageEmbedder(Dinov2Encoder(Dinov2Config.from_dict(raw), WeightMap.from_dir(path), device=device))
    if raw.get("model_type") in ("siglip2", "siglip2_vision_model"):
        from .models.vit import Siglip2Encoder
        return ImageEmbedder(Siglip2Encoder(VisionConfig.from_dict(raw), WeightMap.from_dir(path), device=device))
    if raw.get("model_type") == "dinov3_vit":
        return ImageEmbedder(Dinov3Encoder(Dinov3Config.from_dict(raw), WeightMap.from_dir(path), device=device))
    cfg = VisionConfig.from_dict(raw)
    return ImageEmbedder(VisionEncoder(cfg, WeightMap.from_dir(path), device=device))


class CLIP:
    """Text and image embeddings in one space, plus zero-shot labels."""

    def __init__(self, model, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer
        self.images = ImageEmbedder(model.vision)

    def _ids(self, texts):
        if texts and isinstance(texts[0], str):
            if self.tokenizer is None:
                raise ValueError("string inputs need a tokenizer")
            return self.tokenizer(list(texts), padding="max_length", truncation=True, return_tensors="pt")["input_ids"]
        return torch.tensor(texts)

    def embed_text(self, texts) -> torch.Tensor:
        return self.model.embed_text(self._ids(texts))

    def embed_image(self, images) -> torch.Tensor:
        return self.images.embed(images)

    def zero_shot(self, images, labels) -> torch.Tensor:
        """[images, labels] probabilities (softmax over the labels)."""
        px = self.images.pixels(images if isinstance(images, (list, tuple)) else [images])
        return self.model.logits_per_image(px, self._ids(labels)).softmax(-1)


def load_clip(model: str, *, device: str | torch.device = "cuda") -> CLIP:
    """Full CLIP checkpoint (text + vision towers, projections, logit scale)."""
    import json
    from .models.clip import CLIPDualEncoder
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local CLIP checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        cfg = json.load(f)
    tok = None
    if any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "vocab.json")):
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    return CLIP(CLIPDualEncoder(cfg, WeightMap.from_dir(path), device=device), tok)


class VLM:
    """A vision-language model (``models/llava.py``) plus its serving engine:
    prompts are token ids whose image placeholder runs (one placeholder per
    image token, as the model's processor expands them) receive the images'
    projected features."""

    def __init__(self, vlm, engine_config: EngineConfig | None = None, tokenizer=None):
        import dataclasses
        self.vlm = vlm
        ec = dataclasses.replace(engine_config or EngineConfig(), prefix_caching=False)
        self.engine = LLMEngine(vlm.lm, ec)
        self.tokenizer = tokenizer

    @property
    def image_tokens(self) -> int:
        """Placeholders per image."""
        c = self.vlm.cfg.vision
        n = (c.image_size // c.patch_size) ** 2
        return n + (1 if self.vlm.cfg.vision_feature_select_strategy == "full" else 0)

    def pixels(self, images) -> torch.Tensor:
        return ImageEmbedder(self.vlm.vision).pixels(list(images))

    def generate(self, prompts: list[list[int]], images: list, params: SamplingParams | None = None
                 ) -> list[RequestOutput]:
        """``images[i]``: the images of prompt i (paths, PIL images, HWC uint8
        arrays, or a preprocessed [n, 3, S, S] tensor), in placeholder order."""
        mm = []
        for ids, ims in zip(prompts, images):
            if ims is None or len(ims) == 0:
                mm.append(None)
                continue
            if hasattr(self.vlm, "segments_for_images"):  # NaFlex towers take the images themselves
                mm.append(self.vlm.segments_for_images(list(ids), ims))
                continue
            px = ims if torch.is_tensor(ims) else self.pixels(ims)
            mm.append(self.vlm.mm_segments(list(ids), px))
        return self.engine.generate([list(p) for p in prompts], params, mm)


class AudioLLM:
    """An audio LLM (Voxtral: ``models/voxtral.py``) plus its serving engine:
    prompts are token ids with one audio placeholder per audio token; each
    prompt's audio (16 kHz PCM, or log-mel windows [n, n_mels, frames]) fills
    its placeholders in order."""

    def __init__(self, model, engine_config: EngineConfig | None = None, tokenizer=None):
        import dataclasses
        self.model = model
        ec = dataclasses.replace(engine_config or EngineConfig(), prefix_caching=False)
        self.engine = LLMEngine(model.lm, ec)
        self.tokenizer = tokenizer

    def features(self, audio) -> torch.Tensor:
        """16 kHz PCM -> log-mel windows of 30 s [n, n_mels, 3000] (Voxtral); the
        24 kHz waveform itself for models whose encoders take raw audio (VibeVoice-ASR)."""
        if getattr(self.model, "takes_waveform", False):
            return torch.as_tensor(audio, dtype=torch.float32).reshape(1, -1)
        from .models.whisper import CHUNK_SECONDS, SAMPLE_RATE, log_mel
        a = torch.as_tensor(audio, dtype=torch.float32).flatten()
        n = SAMPLE_RATE * CHUNK_SECONDS
        wins = [a[i:i + n] for i in range(0, max(1, a.numel()), n)]
        return torch.stack([log_mel(w, self.model.cfg.audio.num_mel_bins) for w in wins])

    def generate(self, prompts: list[list[int]], audio: list, params: SamplingParams | None = None
                 ) -> list[RequestOutput]:
        mm = []
        for ids, a in zip(prompts, audio):
            if a is None:
                mm.append(None)
                continue
            mel = a if torch.is_tensor(a) and a.dim() == 3 else self.features(a)
            mm.append(self.model.mm_segments(list(ids), mel))
        return self.engine.generate([list(p) for p in prompts], params, mm)


def load_audio_llm(model: str, *, device: str | torch.device = "cuda",
                   engine_config: EngineConfig | None = None) -> AudioLLM:
    """Voxtral checkpoint (local dir / offline HF id) -> ``AudioLLM``."""
    import json
    from .models.voxtral import VoxtralConfig, VoxtralModel
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    if raw.get("model_type") == "vibevoice_asr":
        from .models.vibevoice import VibeVoiceAsr, VibeVoiceAsrConfig
        m = VibeVoiceAsr(VibeVoiceAsrConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    elif raw.get("model_type") != "voxtral":
        raise NotImplementedError(f"audio LLM model_type {raw.get('model_type')!r}")
    else:
        m = VoxtralModel(VoxtralConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    tok = None
    try:
        from .tokenizer import load_tokenizer
        tok = load_tokenizer(path)
    except Exception:
        pass
    return AudioLLM(m, engine_config, tok)


def load_vlm(model: str, *, device: str | torch.device = "cuda", engine_config: EngineConfig | None = None) -> VLM:
    """LLaVA-form or LFM2-VL vision-language checkpoint (local dir / offline HF id) -> ``VLM``."""
    import json
    from .models.llava import LlavaConfig, LlavaVLM
    path = resolve_model_path(model)
    if path is None:
        raise FileNotFoundError(f"no local checkpoint for {model!r}")
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    if raw.get("model_type") == "lfm2_vl":
        from .models.lfm2_vl import Lfm2VlConfig, Lfm2VlModel
        vlm = Lfm2VlModel(Lfm2VlConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    elif raw.get("model_type") == "llava":
        vlm = LlavaVLM(LlavaConfig.from_dict(raw), WeightMap.from_dir(path), device=device)
    elif raw.get("model_type") == "mistral3":  # Pixtral tower at native image sizes
        from .models.pixtral import Mistral3Config, Mistral3VLM
        vlm = Mistral3VLM(Mistral3Config.from_dict(raw), WeightMap.from_dir(path), device=device)
    else:
        raise NotImplementedError(f"vision-language model_type {raw.get('model_type')!r}")
    tok = None
    try:
        from .tokenizer import load_tokenizer
        tok = load_tokenizer(path)
    except Exception:
        pass
    return VLM(vlm, engine_config, tok)
