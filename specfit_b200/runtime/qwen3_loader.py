"""``load_offloaded_qwen3``: a real Qwen3-MoE checkpoint on the B200 path.

The reference loader (``src/specfit/runtime/qwen3_offloaded_model.py:667-840``)
reads a Hugging Face model directory (``config.json`` plus safetensors
shards), keeps every routed expert in page-locked host memory behind one
``GpuExpertCache`` per layer, and materialises the rest of the model on the
GPU.  This loader does the same for the B200 path: the expert weights of all
layers are packed into one ``ExpertHostPool`` (``[layers, experts, 3*H*I]``
bf16, ``gate | up | down`` rows -- the slot layout the kernels read), every
``layer.mlp`` becomes ``Qwen3B200SparseMoeBlock`` (router + offloaded
experts), and the non-expert parameters are copied to the device from the
shards.

Both expert layouts found in safetensors files are read: one tensor per
expert and projection (``...mlp.experts.{e}.{gate,up,down}_proj.weight``,
the released Qwen3-MoE checkpoints) and the fused per-layer tensors of
transformers 5 (``...mlp.experts.gate_up_proj [E, 2I, H]``, gate rows first,
and ``...mlp.experts.down_proj [E, H, I]``).

Packed-v1 checkpoints (``packed_checkpoint_root``; the reference's
``adapters/qwen3_packed_checkpoint.py``) are read too: ``manifest.json``
(schema ``specfit.qwen3_packed_checkpoint`` version 1), one safetensors file
per layer holding the tensor ``experts [E, 3*H*I]`` in the same
``gate | up | down`` rows, and ``nonexperts.safetensors``.  Their experts are
either copied into a pinned pool (``pinned_copy``) or, the default as in the
reference, used in place: each layer file is memory-mapped and the mapped
tensor registered with ``cudaHostRegister`` (``registered_mmap``), so the
cache fills DMA straight from the page cache.
"""
from __future__ import annotations

import hashlib
import json
import re
import struct
from dataclasses import dataclass
from pathlib import Path

import torch

from .qwen3_offloaded_experts import ExpertExecutionPolicy, ReductionMode

_EXPERT_RE = re.compile(r"^model\.layers\.(\d+)\.mlp\.experts\.(?:(\d+)\.(gate_proj|up_proj|down_proj)\.weight"
                        r"|(gate_up_proj|down_proj))$")


def checkpoint_files(root) -> dict:
    """Tensor name -> safetensors file of a Hugging Face model directory
    (``model.safetensors.index.json`` when sharded, else the single
    ``model.safetensors``)."""
    root = Path(root)
    index = root / "model.safetensors.index.json"
    if index.exists():
        weight_map = json.loads(index.read_text())["weight_map"]
        return {name: root / fname for name, fname in weight_map.items()}
    single = root / "model.safetensors"
    if not single.exists():
        raise FileNotFoundError(f"no safetensors checkpoint under {root}")
    from safetensors import safe_open

    with safe_open(str(single), framework="pt", device="cpu") as f:
        return {name: single for name in f.keys()}


def is_expert_tensor(name: str) -> bool:
    return _EXPERT_RE.match(name) is not None


class _Shards:
    """Open safetensors files by path, reading tensors on the CPU."""

    def __init__(self, files: dict) -> None:
        self.files = files
        self._open: dict = {}

    def get(self, name: str) -> torch.Tensor:
        from safetensors import safe_open

        path = self.files[name]
        f = self._open.get(path)
        if f is None:
            f = self._open[path] = safe_open(str(path), framework="pt", device="cpu")
        return f.get_tensor(name)

    def __contains__(self, name: str) -> bool:
        return name in self.files


def read_expert_layer(shards: _Shards, layer: int, experts: int, hidden: int, inter: int,
                      out: torch.Tensor) -> None:
    """Pack layer ``layer``'s experts into ``out [experts, 3*H*I]``: per expert
    ``gate [I, H] | up [I, H] | down [H, I]`` flattened, cast to ``out``'s dtype."""
    hi = hidden * inter
    fused = f"model.layers.{layer}.mlp.experts.gate_up_proj"
    if fused in shards:
        gu = shards.get(fused)
        dn = shards.get(f"model.layers.{layer}.mlp.experts.down_proj")
        if gu.shape != (experts, 2 * inter, hidden) or dn.shape != (experts, hidden, inter):
            raise ValueError(f"layer {layer}: fused expert tensors have unexpected shapes")
        out[:, : 2 * hi].copy_(gu.reshape(experts, 2 * hi))
        out[:, 2 * hi:].copy_(dn.reshape(experts, hi))
        return
    for e in range(experts):
        base = f"model.layers.{layer}.mlp.experts.{e}"
        parts = []
        for proj, shape in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)),
                            ("down_proj", (hidden, inter))):
            name = f"{base}.{proj}.weight"
            if name not in shards:
                raise KeyError(f"checkpoint has no {name}")
            t = shards.get(name)
            if tuple(t.shape) != shape:
                raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {shape}")
            parts.append(t.reshape(-1))
        out[e].copy_(torch.cat(parts))


def nonexpert_names(files: dict) -> list:
    """Every checkpoint tensor that is not a routed expert weight."""
    return sorted(n for n in files if not is_expert_tensor(n))


PACKED_SCHEMA = "specfit.qwen3_packed_checkpoint"
PACKED_VERSION = 1
PACKED_LAYOUT = ("gate_proj", "up_proj", "down_proj")


class PackedCheckpointError(ValueError):
    """A packed-v1 checkpoint that does not match its manifest."""


@dataclass(frozen=True)
class PackedCheckpoint:
    root: Path
    manifest: dict
    num_layers: int
    num_experts: int
    hidden_size: int
    moe_intermediate_size: int
    packed_elements: int
    layer_files: tuple
    nonexpert_file: Path


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


def _check_file_record(rec: dict, label: str) -> None:
    """One ``files`` record of a packed-v1 manifest: a relative file name that
    stays under the checkpoint root, a positive integer size and a lowercase
    SHA-256 (the record rules of qwen3_packed_checkpoint.py:466-486 and its
    field validators :391-430, same messages)."""
    name = rec.get("filename")
    if not isinstance(name, str) or not name:
        raise PackedCheckpointError("packed checkpoint manifest field 'filename' must be a nonempty string")
    rel = Path(name)
    if rel.is_absolute() or ".." in rel.parts or rel == Path("."):
        raise PackedCheckpointError(f"packed checkpoint {label} file name must stay under root")
    digest = rec.get("sha256")
    if not isinstance(digest, str) or not digest:
        raise PackedCheckpointError("packed checkpoint manifest field 'sha256' must be a nonempty string")
    if len(digest) != 64 or any(c not in "0123456789abcdef" for c in digest):
        raise PackedCheckpointError("packed checkpoint manifest field 'sha256' must be a lowercase SHA256")
    size = rec.get("size_bytes")
    if type(size) is not int or size <= 0:
        raise PackedCheckpointError("packed checkpoint manifest field 'size_bytes' must be a positive integer")


def open_packed_checkpoint(root, *, verify_hashes: bool = False,
                           source_metadata_root=None) -> PackedCheckpoint:
    """Read and check a packed-v1 manifest: the checks of the reference's
    ``PackedQwen3Checkpoint.open`` (qwen3_packed_checkpoint.py:156-377) that
    a loader depends on, with its error type and messages -- schema and
    version, completeness, expert layout and dtype, the packed element
    count, one record per layer in order with the packed shape, file records
    (names under the root, positive sizes, well-formed SHA-256), unique file
    names, file presence and sizes, optionally every file's SHA-256, and,
    with ``source_metadata_root``, that its ``config.json`` and
    ``model.safetensors.index.json`` both exist and are the ones packed.
    Only bf16 experts are accepted (the kernels' dtype)."""
    root = Path(root).resolve()
    mpath = root / "manifest.json"
    if not mpath.is_file():
        raise PackedCheckpointError(f"packed checkpoint manifest is missing: {mpath}")
    try:
        manifest = json.loads(mpath.read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as error:
        raise PackedCheckpointError(f"packed checkpoint manifest is unreadable: {mpath}") from error
    if not isinstance(manifest, dict):
        raise PackedCheckpointError("packed checkpoint manifest must be an object")
    if manifest.get("complete") is not True:
        raise PackedCheckpointError("packed checkpoint manifest must declare complete=true")
    if manifest.get("schema") != PACKED_SCHEMA:
        raise PackedCheckpointError("packed checkpoint manifest schema does not match")
    if manifest.get("schema_version") != PACKED_VERSION:
        raise PackedCheckpointError("packed checkpoint manifest schema version does not match")
    try:
        model = manifest["model"]
        census = model["census"]
        L, E = int(census["num_hidden_layers"]), int(census["num_experts"])
        H, I = int(census["hidden_size"]), int(census["moe_intermediate_size"])
        packed = int(model["packed_expert_elements"])
        files = manifest["files"]
        layers = files["layers"]
        nonexp = files["nonexperts"]
        source = manifest.get("source", {})
    except (KeyError, TypeError, ValueError) as error:
        raise PackedCheckpointError("packed checkpoint manifest lacks model or file records") from error
    dtype = model.get("expert_dtype")
    if dtype != "BF16":
        raise PackedCheckpointError(f"unsupported packed expert dtype: {dtype}")
    if model.get("expert_layout") != list(PACKED_LAYOUT):
        raise PackedCheckpointError("packed checkpoint expert layout does not match")
    if packed != 3 * H * I:
        raise PackedCheckpointError("packed expert element count does not match model dimensions")
    if not isinstance(layers, list):
        raise PackedCheckpointError("packed checkpoint layer files must be a list")
    if len(layers) != L:
        raise PackedCheckpointError("packed checkpoint layer file count does not match census")
    for l, rec in enumerate(layers):
        if not isinstance(rec, dict):
            raise PackedCheckpointError("packed checkpoint layer file record must be an object")
        if rec.get("layer_id") != l:
            raise PackedCheckpointError("packed checkpoint layer IDs must be contiguous")
        if rec.get("tensor_name") != "experts":
            raise PackedCheckpointError("packed checkpoint layer tensor name must be experts")
        if rec.get("shape") != [E, packed]:
            raise PackedCheckpointError("packed checkpoint layer tensor shape does not match")
        if rec.get("dtype") != dtype:
            raise PackedCheckpointError("packed checkpoint layer tensor dtype does not match")
    if not isinstance(nonexp, dict):
        raise PackedCheckpointError("packed checkpoint nonexperts file record must be an object")
    records = [(nonexp, "nonexperts")] + [(rec, f"layer {l}") for l, rec in enumerate(layers)]
    for rec, label in records:
        _check_file_record(rec, label)
    names = [rec["filename"] for rec, _ in records]
    if len(names) != len(set(names)):
        raise PackedCheckpointError("packed checkpoint file names must be unique")
    for rec, _ in records:
        path = root / rec["filename"]
        if not path.is_file():
            raise PackedCheckpointError(f"packed checkpoint file is missing: {path}")
        if path.stat().st_size != rec["size_bytes"]:
            raise PackedCheckpointError(f"packed checkpoint file size does not match: {path}")
        if verify_hashes and _sha256(path) != rec["sha256"]:
            raise PackedCheckpointError(f"packed checkpoint file SHA256 does not match: {path}")
    if source_metadata_root is not None:
        meta = Path(source_metadata_root).resolve()
        cfg, index = meta / "config.json", meta / "model.safetensors.index.json"
        if not cfg.is_file() or not index.is_file():
            raise PackedCheckpointError("source config or index metadata is missing")
        if _sha256(cfg) != source.get("config_sha256"):
            raise PackedCheckpointError("source config SHA256 does not match packed checkpoint")
        if _sha256(index) != source.get("index_sha256"):
            raise PackedCheckpointError("source index SHA256 does not match packed checkpoint")
    return PackedCheckpoint(root, manifest, L, E, H, I, packed,
                            tuple(root / r["filename"] for r in layers), root / nonexp["filename"])


def _safetensors_span(path: Path, name: str) -> tuple:
    """(byte offset, byte length, dtype, shape) of tensor ``name`` in a
    safetensors file: an 8-byte little-endian header size, a JSON header with
    each tensor's ``data_offsets`` relative to the data that follows it."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    if name not in header:
        raise PackedCheckpointError(f"{path} has no tensor {name!r}")
    meta = header[name]
    begin, end = meta["data_offsets"]
    return 8 + n + begin, end - begin, meta["dtype"], tuple(meta["shape"])


def map_packed_layer(path: Path, experts: int, packed: int) -> torch.Tensor:
    """The ``experts`` tensor of a packed layer file as a bf16 view of a
    private memory mapping of the file (no copy)."""
    off, nbytes, dtype, shape = _safetensors_span(path, "experts")
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if set(json.loads(f.read(n))) - {"__metadata__"} != {"experts"}:
            raise PackedCheckpointError(f"packed expert layer must contain only 'experts': {path}")
    if dtype != "BF16" or shape != (experts, packed) or nbytes != experts * packed * 2:
        raise PackedCheckpointError(f"{path}: experts tensor is not BF16 [{experts}, {packed}]")
    size = path.stat().st_size
    raw = torch.from_file(str(path), shared=False, size=size, dtype=torch.uint8)
    return raw[off: off + nbytes].view(torch.bfloat16).view(experts, packed)


_HOST_REGISTER_READ_ONLY = 0x08 | 0x02 | 0x01  # read-only (never written), mapped for kernels, portable


class MappedExpertPool:
    """Expert sources in place in a packed-v1 checkpoint: one memory-mapped
    ``[E, 3*H*I]`` tensor per layer, each registered read-only with
    ``cudaHostRegister`` (the reference's ``RegisteredMmapExpertLayer``,
    runtime/registered_mmap.py:12-97), with the ``sources`` / ``close``
    interface of ``ExpertHostPool``."""

    def __init__(self, ckpt: PackedCheckpoint, device) -> None:
        self.layers = [map_packed_layer(p, ckpt.num_experts, ckpt.packed_elements) for p in ckpt.layer_files]
        self.experts = ckpt.num_experts
        self.device = torch.device(device)
        self._registered = []
        with torch.cuda.device(self.device):
            for t in self.layers:
                # The whole file mapping is registered: torch judges a view
                # pinned by its storage's base address, and the expert tensor
                # starts after the safetensors header inside that storage.
                store = t.untyped_storage()
                rc = int(torch.cuda.cudart().cudaHostRegister(store.data_ptr(), store.nbytes(),
                                                              _HOST_REGISTER_READ_ONLY))
                if rc != 0:
                    self.close()
                    raise RuntimeError(f"cudaHostRegister of a packed expert layer failed ({rc})")
                self._registered.append(store)
                if not t.is_pinned():
                    self.close()
                    raise RuntimeError("a registered packed expert layer is not seen as pinned memory")

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.layers)

    def sources(self, layer: int) -> dict:
        from .state import ExpertKey

        return {ExpertKey(layer, e): self.layers[layer][e] for e in range(self.experts)}

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for store in self._registered:
                torch.cuda.cudart().cudaHostUnregister(store.data_ptr())
        self._registered = []


def load_offloaded_qwen3(model_root, *, device, slots_per_layer: int, packed_checkpoint_root=None,
                         packed_expert_backing=None, verify_packed_hashes: bool = False,
                         reduction_mode=ReductionMode.CANONICAL,
                         expert_execution_policy=ExpertExecutionPolicy.EXPERT_ID_ASCENDING,
                         attn_implementation: str = "sdpa", cache_observer=None,
                         h2d_prefetch: bool = True):
    """Load a Hugging Face Qwen3-MoE directory as a ``LoadedOffloadedQwen3``
    (same arguments and validation as the reference's loader).  With
    ``attn_implementation="sdpa"`` (the reference's default and requirement
    for tree verification) attention runs on the tree-attention kernel; any
    other registered implementation name is passed to transformers."""
    from transformers import GenerationConfig, Qwen3MoeConfig, Qwen3MoeForCausalLM

    from .gpu_expert_cache import GpuExpertCache
    from .moe_block import Qwen3B200SparseMoeBlock, Qwen3B200TopKRouter
    from .qwen3_offloaded_experts import Qwen3OffloadedExperts
    from .qwen3_verifier import ExpertHostPool, LoadedB200Qwen3
    from .tree_attention import install as install_tree_attention

    if type(h2d_prefetch) is not bool:
        raise ValueError("h2d_prefetch must be a boolean")
    policy = ExpertExecutionPolicy(expert_execution_policy)
    reduction = ReductionMode(reduction_mode)
    if packed_expert_backing is None:
        backing = "registered_mmap" if packed_checkpoint_root is not None else "pinned_copy"
    else:
        backing = getattr(packed_expert_backing, "value", packed_expert_backing)
    if backing not in ("pinned_copy", "registered_mmap"):
        raise ValueError(f"unknown packed expert backing {packed_expert_backing!r}")
    if packed_checkpoint_root is None and backing != "pinned_copy":
        raise ValueError("registered_mmap requires packed_checkpoint_root")
    root = Path(model_root).resolve()
    packed = (open_packed_checkpoint(packed_checkpoint_root, verify_hashes=verify_packed_hashes,
                                     source_metadata_root=root)
              if packed_checkpoint_root is not None else None)
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("offloaded Qwen3 requires a CUDA device")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    cfg = Qwen3MoeConfig.from_pretrained(root, local_files_only=True)
    if cfg.hidden_act != "silu":
        raise ValueError("P0 loader requires hidden_act='silu'")
    if not 1 <= slots_per_layer <= cfg.num_experts:
        raise ValueError(f"slots_per_layer must be in [1, {cfg.num_experts}]")
    if cfg.mlp_only_layers or getattr(cfg, "decoder_sparse_step", 1) != 1:
        raise ValueError("P0 loader requires an MoE block in every layer")
    # The model's config keeps the requested implementation ("sdpa" by
    # default, which the reference speculator requires); with "sdpa" the
    # decoder layers' attention is then routed to the tree kernel.
    cfg._attn_implementation = attn_implementation

    L, E = cfg.num_hidden_layers, cfg.num_experts
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    if packed is not None:
        if (packed.num_layers, packed.num_experts, packed.hidden_size, packed.moe_intermediate_size) != (L, E, H, I):
            raise PackedCheckpointError("packed checkpoint census differs from config.json")
        from safetensors import safe_open

        with safe_open(str(packed.nonexpert_file), framework="pt", device="cpu") as f:
            files = {name: packed.nonexpert_file for name in f.keys()}
        shards = _Shards(files)
        if backing == "registered_mmap":
            pool = MappedExpertPool(packed, dev)
        else:
            pool = ExpertHostPool(L, E, 3 * H * I, torch.bfloat16)
            for layer in range(L):
                pool.data[layer].copy_(map_packed_layer(packed.layer_files[layer], E, 3 * H * I))
    else:
        files = checkpoint_files(root)
        shards = _Shards(files)
        pool = ExpertHostPool(L, E, 3 * H * I, torch.bfloat16)
        for layer in range(L):
            read_expert_layer(shards, layer, E, H, I, pool.data[layer])

    with torch.device("meta"):
        model = Qwen3MoeForCausalLM(cfg)
    caches = []
    for l, layer in enumerate(model.model.layers):
        cache = GpuExpertCache(pool.sources(l), slot_count=slots_per_layer, device=dev,
                               adopt_pinned_sources=True, observer=cache_observer)
        experts = Qwen3OffloadedExperts(layer_id=l, cache=cache, hidden_size=H, intermediate_size=I,
                                        reduction_mode=reduction, execution_policy=policy,
                                        h2d_prefetch=h2d_prefetch)
        gate = Qwen3B200TopKRouter(E, H, cfg.num_experts_per_tok, cfg.norm_topk_prob, device="meta")
        layer.mlp = Qwen3B200SparseMoeBlock(gate, experts)
        caches.append(cache)
    model.to_empty(device=dev)
    params = dict(model.named_parameters())
    names = nonexpert_names(files)
    missing = sorted(set(params) - set(names))
    if cfg.tie_word_embeddings and missing == ["lm_head.weight"]:
        missing = []
    if missing:
        raise KeyError(f"checkpoint lacks parameters: {missing[:5]}")
    with torch.no_grad():
        for name in names:
            if name not in params:
                continue  # e.g. buffers saved by other versions
            t = shards.get(name)
            p = params[name]
            if tuple(t.shape) != tuple(p.shape):
                raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(p.shape)}")
            p.data = t.to(device=dev, dtype=torch.bfloat16)
        if cfg.tie_word_embeddings:
            model.lm_head.weight = model.model.embed_tokens.weight
    # RoPE frequencies in fp32, built on the device (as a model loaded in bf16 keeps them).
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg, device=dev)
    if (root / "generation_config.json").exists():
        model.generation_config = GenerationConfig.from_pretrained(root, local_files_only=True)
    if attn_implementation == "sdpa":
        install_tree_attention(model)
    model.requires_grad_(False)
    model.eval()
    torch.cuda.synchronize(dev)
    return LoadedB200Qwen3(model, tuple(caches), pool)
