"""Offline model utilities: norm tweaking, pruning, LoRA merge, hub resolution, capabilities."""
