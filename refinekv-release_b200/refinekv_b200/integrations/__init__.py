"""Model-framework adapters (imported lazily: ``refinekv_b200.RefineKV``)."""
