"""Continuous-integration support: test shards (``shards``), a resource
sampler for test and bench runs (``resource_sampler``) and repository policy
checks (``policy``). The workflow in ``.github/workflows/ci.yml`` drives
them."""
