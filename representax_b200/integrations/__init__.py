from .huggingface import load_hf_config, load_safetensor_subset, resolve_hf_checkpoint, save_safetensors

__all__ = ["load_hf_config", "load_safetensor_subset", "resolve_hf_checkpoint", "save_safetensors"]
