"""Model definitions, sharding rules, synthetic weights and the on-disk artifact format."""
