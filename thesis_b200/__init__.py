"""B200-native packed LayerSkip-Llama draft/verify step (see DESIGN.md at the repository root)."""
