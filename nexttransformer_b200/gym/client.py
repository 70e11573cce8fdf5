"""Python client of the gym HTTP API (the MCP adapter uses it too)."""
import json
from pathlib import Path

import requests

from nexttransformer_b200.gym.contract import SCHEMA_VERSION, GymError


class GymClient:
    def __init__(self, endpoint, token, timeout=600):
        self.endpoint, self.token, self.timeout = endpoint.rstrip("/"), token, timeout

    @classmethod
    def from_credential(cls, path):
        """Client from a credential file ``{"endpoint", "token"}``."""
        c = json.loads(Path(path).read_text())
        return cls(c["endpoint"], c["token"])

    def call(self, operation, **params):
        r = requests.post(f"{self.endpoint}/v1/call", timeout=self.timeout,
                          headers={"Authorization": f"Bearer {self.token}"},
                          json=dict(schema_version=SCHEMA_VERSION, operation=operation, params=params))
        body = r.json()
        if "error" in body:
            raise GymError(body["error"]["code"], body["error"]["message"], r.status_code)
        return body["result"]
