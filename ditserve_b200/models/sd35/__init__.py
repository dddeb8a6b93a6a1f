"""SD3.5-Medium MMDiT: model, continuous-batching engine, worker backend."""
