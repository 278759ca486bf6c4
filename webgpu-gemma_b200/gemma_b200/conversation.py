"""Gemma chat template with optional tool declarations (restates src/conversation.ts:6-52)."""
from __future__ import annotations

import json


def build_chat_prompt(history: list[dict], tools_json: str | None = None) -> str:
    system_prefix = ""
    tools = None
    try:
        if tools_json:
            parsed = json.loads(tools_json)
            if isinstance(parsed, list) and parsed:
                tools = parsed
    except (ValueError, TypeError):
        tools = None
    if tools:
        decl = ""
        for tool in tools:
            decl += f"<start_function_declaration>declaration:{tool.get('name')}{{"
            decl += f"description:<escape>{tool.get('description')}<escape>"
            params = tool.get("parameters")
            if params:
                decl += ",parameters:{properties:{"
                props = (params.get("properties") or {}).items()
                items = []
                for k, v in props:
                    p = f"{k}:{{description:<escape>{v.get('description')}<escape>,type:<escape>{v.get('type')}<escape>"
                    if v.get("enum"):
                        p += ",enum:[" + ",".join(f"<escape>{e}<escape>" for e in v["enum"]) + "]"
                    p += "}"
                    items.append(p)
                decl += ",".join(items) + "}"
                if params.get("required"):
                    decl += ",required:[" + ",".join(f"<escape>{r}<escape>" for r in params["required"]) + "]"
                decl += f",type:<escape>{params.get('type')}<escape>"
                decl += "}"
            decl += "}<end_function_declaration>"
        system_prefix = ("<start_of_turn>developer\nYou are a model that can do function calling with the "
                         f"following functions\n{decl}\n<end_of_turn>\n")
    prompt = system_prefix
    for turn in history:
        prompt += f"<start_of_turn>{turn['role']}\n{turn['text']}<end_of_turn>\n"
    return prompt + "<start_of_turn>model\n"
