// TypeScript client of the openmini_v1_b200 HTTP API (fetch-based, no dependencies;
// Node >= 18 or any browser). Covers the OpenAI-compatible routes, the /api/v1 routes
// and the admin API's login.
//
// Reference counterpart: openmini-server/bindings/*.ts (typed wrappers of the same
// service); the request / response field names follow this server's handlers in
// openmini_v1_b200/serve/http.py.

export interface CompletionRequest {
  prompt: string | number[];
  max_tokens?: number;
  temperature?: number;
  top_p?: number;
  top_k?: number;
  stop?: string[];
  seed?: number;
}

export interface CompletionChoice {
  index: number;
  text: string;
  token_ids: number[];
  finish_reason: string | null;
}

export interface Usage {
  prompt_tokens: number;
  completion_tokens: number;
  total_tokens?: number;
}

export interface CompletionResponse {
  id: string;
  object: string;
  created: number;
  model: string;
  choices: CompletionChoice[];
  usage: Usage;
}

export interface ChatMessage {
  role: "system" | "user" | "assistant";
  content: string;
}

export interface ChatResponse {
  session_id: string;
  response: string;
  finish_reason: string | null;
  usage: Usage;
}

export interface ImageAnswer {
  answer: string;
  usage: Usage;
}

export interface SpeechAudio {
  audio_data: string;   // base64 WAV (16-bit PCM mono)
  sample_rate: number;
  duration_s: number;
}

export interface Transcript {
  text: string;
  tokens: number;
}

export class OpenMiniError extends Error {
  constructor(public status: number, body: string) {
    super(`openmini HTTP ${status}: ${body}`);
  }
}

export class OpenMiniClient {
  private token?: string;

  constructor(private baseUrl = "http://127.0.0.1:8080", private timeoutMs = 120_000) {}

  private async call<T>(method: string, path: string, body?: unknown): Promise<T> {
    const ctl = new AbortController();
    const timer = setTimeout(() => ctl.abort(), this.timeoutMs);
    try {
      const headers: Record<string, string> = { "Content-Type": "application/json" };
      if (this.token) headers["Authorization"] = `Bearer ${this.token}`;
      const r = await fetch(this.baseUrl + path, {
        method, headers, body: body === undefined ? undefined : JSON.stringify(body), signal: ctl.signal,
      });
      if (!r.ok) throw new OpenMiniError(r.status, await r.text());
      return (await r.json()) as T;
    } finally {
      clearTimeout(timer);
    }
  }

  health(): Promise<Record<string, unknown>> {
    return this.call("GET", "/health");
  }

  models(): Promise<{ data: { id: string }[] }> {
    return this.call("GET", "/v1/models");
  }

  complete(req: CompletionRequest): Promise<CompletionResponse> {
    return this.call("POST", "/v1/completions", { ...req, stream: false });
  }

  /** Server-sent events of /v1/completions with stream = true: yields each text piece. */
  async *completeStream(req: CompletionRequest): AsyncGenerator<string> {
    const r = await fetch(this.baseUrl + "/v1/completions", {
      method: "POST", headers: { "Content-Type": "application/json" }, body: JSON.stringify({ ...req, stream: true }),
    });
    if (!r.ok || !r.body) throw new OpenMiniError(r.status, await r.text());
    const reader = r.body.getReader();
    const dec = new TextDecoder();
    let buf = "";
    for (;;) {
      const { value, done } = await reader.read();
      if (done) break;
      buf += dec.decode(value, { stream: true });
      let i: number;
      while ((i = buf.indexOf("\n\n")) >= 0) {
        const ev = buf.slice(0, i);
        buf = buf.slice(i + 2);
        if (!ev.startsWith("data: ")) continue;
        const data = ev.slice(6);
        if (data === "[DONE]") return;
        const j = JSON.parse(data);
        yield j.choices?.[0]?.text ?? "";
      }
    }
  }

  chat(messages: ChatMessage[], opts: { max_tokens?: number; temperature?: number; session_id?: string } = {}):
      Promise<ChatResponse> {
    return this.call("POST", "/api/v1/chat", { messages, ...opts });
  }

  imageUnderstand(imageBytes: Uint8Array, question: string, maxTokens = 0): Promise<ImageAnswer> {
    let bin = "";
    imageBytes.forEach((b) => (bin += String.fromCharCode(b)));
    return this.call("POST", "/api/v1/image/understand", { image: btoa(bin), question, max_tokens: maxTokens });
  }

  textToSpeech(text: string, opts: { voice?: string; language?: string; speed?: number; pitch?: number } = {}):
      Promise<SpeechAudio> {
    return this.call("POST", "/api/v1/tts", { text, ...opts });
  }

  speechToText(wavBytes: Uint8Array, language = "", maxTokens = 0): Promise<Transcript> {
    let bin = "";
    wavBytes.forEach((b) => (bin += String.fromCharCode(b)));
    return this.call("POST", "/api/v1/stt", { audio: btoa(bin), language, max_tokens: maxTokens });
  }

  stats(): Promise<Record<string, unknown>> {
    return this.call("GET", "/api/v1/inference/stats");
  }

  async adminLogin(username: string, password: string): Promise<void> {
    const r = await this.call<{ token: string }>("POST", "/admin/auth/login", { username, password });
    this.token = r.token;
  }

  admin<T = unknown>(path: string, method = "GET", body?: unknown): Promise<T> {
    return this.call(method, "/admin" + path, body);
  }
}
