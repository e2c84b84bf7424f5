"""scalatorch (B200 mirror): host-side Python mirror of scala-torch's Linear / Llama hot path.

Modules mirror the reference's packages: ffm (device session over libstb200.so), nn (Linear),
io (safetensors raw payloads), models (LlamaConfig, BackendLlama).  All arithmetic runs in
libstb200.so on the GPU; this package only validates arguments and moves handles.
"""
from . import ffm  # noqa: F401
