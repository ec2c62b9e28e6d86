"""Data pipeline: corpus builder, token store, cost model, packers, scheduler, loader."""
