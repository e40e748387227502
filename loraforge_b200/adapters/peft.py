"""Local PEFT linear-LoRA checkpoints read into CPU tensors (no PEFT import).

Same file contract and refusal rules as the reference loader
(src/loraforge/adapters/peft.py:117-197, configuration rules in
src/loraforge/adapters/_config.py:1-118): a directory holding
``adapter_config.json`` and a single ``adapter_model.safetensors`` whose keys are
``base_model.model.<module>.lora_{A,B}.weight``; per-module rank and alpha follow
PEFT's ordered suffix-regex ``rank_pattern`` / ``alpha_pattern``; scaling is alpha/r,
or alpha/sqrt(r) with ``use_rslora``.  An optional ``loraforge_manifest.json`` is
checked against the files' SHA-256 digests and sizes.  Anything the serving path
could not reproduce exactly (DoRA, biases, fan-in/fan-out storage, non-default
initialisation schemes, extra saved modules...) is refused rather than dropped.
"""

from __future__ import annotations

import hashlib
import json
import math
import re
from dataclasses import dataclass
from pathlib import Path
from typing import TYPE_CHECKING

if TYPE_CHECKING:
    from torch import Tensor

CONFIG = "adapter_config.json"
WEIGHTS = "adapter_model.safetensors"
MANIFEST = "loraforge_manifest.json"
_KEY = re.compile(r"^base_model\.model\.(.+)\.lora_([AB])\.weight$")

# PEFT LoraConfig fields, split by what the serving path accepts for them.
_MUST_BE_FALSE = ("fan_in_fan_out", "use_dora", "use_qalora", "lora_bias")
_MUST_BE_EMPTY = (
    "modules_to_save",
    "layer_replication",
    "target_parameters",
    "trainable_token_indices",
    "megatron_config",
    "loftq_config",
    "eva_config",
    "corda_config",
    "arrow_config",
    "alora_invocation_tokens",
)
_ACCEPTED = frozenset(
    (
        "peft_type", "task_type", "base_model_name_or_path", "revision", "auto_mapping",
        "inference_mode", "r", "lora_alpha", "use_rslora", "lora_dropout", "bias",
        "target_modules", "exclude_modules", "layers_to_transform", "layers_pattern",
        "rank_pattern", "alpha_pattern", "init_lora_weights", "megatron_core",
        "qalora_group_size", "peft_version", "ensure_weight_tying", "runtime_config",
    )
    + _MUST_BE_FALSE
    + _MUST_BE_EMPTY
)


@dataclass(frozen=True)
class AdapterModule:
    """One LoRA pair: ``a`` [rank, in_features], ``b`` [out_features, rank]."""

    name: str
    a: Tensor
    b: Tensor
    alpha: float
    use_rslora: bool = False

    @property
    def rank(self) -> int:
        return self.a.shape[0]

    @property
    def scaling(self) -> float:
        return self.alpha / (math.sqrt(self.rank) if self.use_rslora else self.rank)


@dataclass(frozen=True)
class PeftAdapter:
    """CPU snapshot of a local adapter directory; treat everything as read-only."""

    source: Path
    config: dict
    modules: tuple[AdapterModule, ...]
    source_sha256: dict[str, str]


def _positive_int(value, name: str) -> int:
    if type(value) is not int or value < 1:
        raise ValueError(f"{name} must be a positive integer")
    return value


def _finite(value, name: str) -> float:
    if type(value) not in (int, float) or not math.isfinite(value):
        raise ValueError(f"{name} must be a finite number")
    return float(value)


def _sha256(path: Path) -> str:
    digest = hashlib.sha256()
    with path.open("rb") as handle:
        while block := handle.read(1 << 20):
            digest.update(block)
    return digest.hexdigest()


def _read_object(path: Path) -> dict:
    def no_duplicates(pairs):
        seen = {}
        for key, value in pairs:
            if key in seen:
                raise ValueError(f"duplicate JSON key in {path.name}: {key}")
            seen[key] = value
        return seen

    data = json.loads(path.read_text(), object_pairs_hook=no_duplicates)
    if not isinstance(data, dict):
        raise ValueError(f"{path.name} must contain a JSON object")
    return data


def check_config(config: dict) -> None:
    """Refuse PEFT configurations whose weights the LoRA path cannot apply exactly."""
    if config.get("peft_type") != "LORA":
        raise ValueError("only PEFT LORA adapters are supported")
    unknown = sorted(set(config) - _ACCEPTED)
    if unknown:
        raise ValueError(f"unsupported configuration fields: {unknown}")
    for field in _MUST_BE_FALSE:
        if config.get(field, False) is not False:
            raise ValueError(f"unsupported LoRA configuration: {field}")
    if type(config.get("use_rslora", False)) is not bool:
        raise ValueError("use_rslora must be a boolean")
    for field in _MUST_BE_EMPTY:
        if config.get(field) not in (None, [], {}):
            raise ValueError(f"unsupported LoRA configuration: {field}")
    if config.get("ensure_weight_tying", False) is not False:
        raise ValueError("ensure_weight_tying is not supported")
    if config.get("runtime_config") not in (None, {}, {"ephemeral_gpu_offload": False}):
        raise ValueError("non-default runtime_config is not supported")
    if config.get("bias", "none") != "none":
        raise ValueError("bias weights are not supported")
    if type(config.get("init_lora_weights", True)) is not bool:
        raise ValueError("special LoRA initialization schemes are not supported")
    _positive_int(config.get("r"), "r")
    _finite(config.get("lora_alpha"), "lora_alpha")
    if not 0 <= _finite(config.get("lora_dropout", 0), "lora_dropout") <= 1:
        raise ValueError("lora_dropout must be between zero and one")
    for field, check in (("rank_pattern", _positive_int), ("alpha_pattern", _finite)):
        patterns = config.get(field, {})
        if not isinstance(patterns, dict):
            raise ValueError(f"{field} must be an object")
        for key, value in patterns.items():
            if not isinstance(key, str) or not key:
                raise ValueError(f"{field} keys must be nonempty strings")
            re.compile(_suffix_regex(key))
            check(value, field)
    targets = config.get("target_modules")
    if not isinstance(targets, (str, list)) or not targets:
        raise ValueError("explicit target_modules are required")
    if isinstance(targets, list) and not all(isinstance(t, str) and t for t in targets):
        raise ValueError("target_modules must contain nonempty strings")


def _suffix_regex(pattern: str) -> str:
    # PEFT matches pattern keys against a module name's dotted suffix.
    return rf"(?:.*\.)?(?:{pattern})"


def pattern_value(patterns: dict, name: str, default):
    """First pattern (in file order) matching ``name``'s suffix, else ``default``."""
    for pattern, value in patterns.items():
        if re.fullmatch(_suffix_regex(pattern), name):
            return value
    return patterns.get(name, default)


def targets_module(targets, name: str) -> bool:
    """PEFT's target test: a full regex for a string, a dotted suffix for a list."""
    if isinstance(targets, str):
        return re.fullmatch(targets, name) is not None
    return any(name == t or name.endswith("." + t) for t in targets or ())


def _check_manifest(directory: Path) -> None:
    path = directory / MANIFEST
    if not path.exists():
        return
    manifest = _read_object(path)
    if (
        type(manifest.get("schema_version")) is not int
        or manifest["schema_version"] != 1
        or manifest.get("format") != "loraforge.peft"
    ):
        raise ValueError("unsupported LoRAForge manifest version or format")
    output = manifest.get("output")
    if not isinstance(output, dict) or not isinstance(output.get("files"), dict):
        raise ValueError("manifest output.files must be an object")
    for name in (CONFIG, WEIGHTS):
        record = output["files"].get(name, {})
        if not isinstance(record, dict):
            raise ValueError(f"manifest file record must be an object: {name}")
        target = directory / name
        if record.get("sha256") != _sha256(target) or record.get("bytes") != target.stat().st_size:
            raise ValueError(f"manifest integrity check failed for {name}")


def load_peft_adapter(directory: str | Path) -> PeftAdapter:
    """Read a local single-file safetensors PEFT adapter into CPU tensors.

    Modules come back sorted by name with cloned factors.  The files are hashed
    before and after parsing; a change in between is an error.
    """
    import torch
    from safetensors.torch import load_file

    source = Path(directory).resolve(strict=True)
    if not source.is_dir() or not all((source / n).is_file() for n in (CONFIG, WEIGHTS)):
        raise ValueError("expected adapter_config.json and adapter_model.safetensors in a directory")
    _check_manifest(source)
    names = [CONFIG, WEIGHTS] + ([MANIFEST] if (source / MANIFEST).exists() else [])
    digests = {name: _sha256(source / name) for name in names}
    config = _read_object(source / CONFIG)
    check_config(config)
    pairs: dict[str, dict[str, Tensor]] = {}
    for key, tensor in load_file(source / WEIGHTS, device="cpu").items():
        match = _KEY.fullmatch(key)
        if match is None:
            raise ValueError(f"unsupported tensor key: {key}")
        if tensor.ndim != 2 or tensor.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError(f"unsupported tensor layout or dtype: {key}")
        module, side = match.groups()
        pairs.setdefault(module, {})[side] = tensor
    if not pairs:
        raise ValueError("adapter has no LoRA tensor pairs")
    modules = []
    for name in sorted(pairs):
        pair = pairs[name]
        if set(pair) != {"A", "B"}:
            raise ValueError(f"incomplete A/B pair: {name}")
        a, b = pair["A"], pair["B"]
        rank = pattern_value(config.get("rank_pattern", {}), name, config["r"])
        alpha = pattern_value(config.get("alpha_pattern", {}), name, config["lora_alpha"])
        if min(*a.shape, *b.shape) < 1 or a.shape[0] != rank or b.shape[1] != rank or a.dtype != b.dtype:
            raise ValueError(f"factor shape/dtype disagrees with configured rank: {name}")
        if not (torch.isfinite(a).all().item() and torch.isfinite(b).all().item()):
            raise ValueError(f"nonfinite factors: {name}")
        if not targets_module(config["target_modules"], name) or targets_module(
            config.get("exclude_modules"), name
        ):
            raise ValueError(f"tensor module disagrees with target/exclude configuration: {name}")
        modules.append(
            AdapterModule(name, a.clone(), b.clone(), float(alpha), config.get("use_rslora", False))
        )
    if any(_sha256(source / name) != digest for name, digest in digests.items()):
        raise ValueError("source adapter changed while it was being read")
    return PeftAdapter(source, config, tuple(modules), digests)


def write_manifest(directory: str | Path) -> dict:
    """Write ``loraforge_manifest.json`` recording the digests of the two adapter files.

    ``load_peft_adapter`` then refuses the directory if either file changes.
    """
    directory = Path(directory)
    files = {
        name: {"sha256": _sha256(directory / name), "bytes": (directory / name).stat().st_size}
        for name in (CONFIG, WEIGHTS)
    }
    manifest = {"format": "loraforge.peft", "schema_version": 1, "output": {"files": files}}
    (directory / MANIFEST).write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest
