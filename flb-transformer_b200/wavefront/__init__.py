"""Wavefront engine (B200 build of FLB-Transformer's wavefront package)."""
from .wavefront_api import WavefrontConfig, generate_wavefront_schedule
from .wavefront_engine import WavefrontEngine, WavefrontEngineFunction
from .wavefront_kernel import fetch_mapped_context, run_fetch_kernel
from .wavefront_graph import GraphedWavefrontEngine

__all__ = ["WavefrontConfig", "generate_wavefront_schedule", "WavefrontEngine",
           "WavefrontEngineFunction", "fetch_mapped_context", "run_fetch_kernel",
           "GraphedWavefrontEngine"]
