"""Seeded synthetic checkpoints (weights, configs, tokenizer) and input batches of the benchmark
configurations, in the reference's file layout and ABI terms. Used by the tests and the benchmarks;
nothing in here computes any part of the model."""
