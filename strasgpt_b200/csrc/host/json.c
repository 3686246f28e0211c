// Recursive-descent JSON reader. See json.h.
#include "json.h"

#include <limits.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  const char* p;
  const char* end;
  size_t line;
  const char* what;
} cursor_t;

static void die_at(const cursor_t* c, const char* msg) {
  fprintf(
      stderr, "[StrasGPT] Error: %s: line %zu: %s\n", c->what, c->line, msg
  );
  exit(EXIT_FAILURE);
}

static void* xrealloc(void* p, size_t n) {
  void* q = realloc(p, n);
  if (!q && n) {
    fprintf(stderr, "[StrasGPT] Error: out of host memory (json)\n");
    exit(EXIT_FAILURE);
  }
  return q;
}

static void skip_space(cursor_t* c) {
  while (c->p < c->end) {
    char ch = *c->p;
    if (ch == '\n') {
      c->line++;
    } else if (ch != ' ' && ch != '\t' && ch != '\r') {
      return;
    }
    c->p++;
  }
}

// Raw string: bytes between the quotes, a backslash escapes the next byte.
static char* parse_string_raw(cursor_t* c) {
  if (c->p >= c->end || *c->p != '"') {
    die_at(c, "expected a string");
  }
  const char* start = ++c->p;
  while (c->p < c->end && *c->p != '"') {
    if (*c->p == '\\') {
      c->p++;
    }
    if (c->p < c->end && *c->p == '\n') {
      c->line++;
    }
    c->p++;
  }
  if (c->p >= c->end) {
    die_at(c, "unterminated string");
  }
  size_t n = (size_t)(c->p - start);
  c->p++; // closing quote
  char* s = malloc(n + 1);
  if (!s) {
    die_at(c, "out of host memory");
  }
  memcpy(s, start, n);
  s[n] = '\0';
  return s;
}

static bool is_digit(char ch) { return ch >= '0' && ch <= '9'; }

// Number with the reference scanner's integer/float split
// (source/json_scanner.l:23-24,58-80): an integer literal is exact; a float
// literal counts as an integer when it has no fractional part.
static void parse_number(cursor_t* c, json_value_t* v) {
  const char* s = c->p;
  const char* q = s;
  if (q < c->end && (*q == '-' || *q == '+')) {
    q++;
  }
  bool any_digit = false;
  while (q < c->end && is_digit(*q)) {
    q++;
    any_digit = true;
  }
  bool is_float = false;
  if (q < c->end && *q == '.') {
    is_float = true;
    q++;
    while (q < c->end && is_digit(*q)) {
      q++;
      any_digit = true;
    }
  }
  if (!any_digit) {
    die_at(c, "malformed number");
  }
  if (q < c->end && (*q == 'e' || *q == 'E')) {
    is_float = true;
    q++;
    if (q < c->end && (*q == '-' || *q == '+')) {
      q++;
    }
    if (q >= c->end || !is_digit(*q)) {
      die_at(c, "malformed exponent");
    }
    while (q < c->end && is_digit(*q)) {
      q++;
    }
  }
  char buf[128];
  size_t n = (size_t)(q - s);
  if (n >= sizeof(buf)) {
    die_at(c, "number literal too long");
  }
  memcpy(buf, s, n);
  buf[n] = '\0';
  v->kind = JSON_NUMBER;
  if (!is_float) {
    v->is_int = true;
    v->ival = atoll(buf);
    v->fval = (double)v->ival;
  } else {
    double d = atof(buf);
    double ip;
    v->fval = d;
    v->is_int = (modf(d, &ip) == 0.0) && d >= (double)LLONG_MIN &&
                d <= (double)LLONG_MAX;
    v->ival = v->is_int ? (long long)d : 0;
  }
  c->p = q;
}

static bool match_word(cursor_t* c, const char* w) {
  size_t n = strlen(w);
  if ((size_t)(c->end - c->p) >= n && memcmp(c->p, w, n) == 0) {
    c->p += n;
    return true;
  }
  return false;
}

static void parse_value(cursor_t* c, json_value_t* v, int depth);

static void parse_container(cursor_t* c, json_value_t* v, int depth) {
  bool object = (*c->p == '{');
  char close = object ? '}' : ']';
  v->kind = object ? JSON_OBJECT : JSON_ARRAY;
  c->p++;
  size_t cap = 0;
  skip_space(c);
  if (c->p < c->end && *c->p == close) {
    c->p++;
    return;
  }
  for (;;) {
    if (v->count == cap) {
      cap = cap ? cap * 2 : 8;
      v->item = xrealloc(v->item, cap * sizeof(*v->item));
      if (object) {
        v->key = xrealloc(v->key, cap * sizeof(*v->key));
      }
    }
    skip_space(c);
    if (object) {
      v->key[v->count] = parse_string_raw(c);
      skip_space(c);
      if (c->p >= c->end || *c->p != ':') {
        die_at(c, "expected ':'");
      }
      c->p++;
    }
    memset(&v->item[v->count], 0, sizeof(v->item[0]));
    parse_value(c, &v->item[v->count], depth + 1);
    v->count++;
    skip_space(c);
    if (c->p < c->end && *c->p == ',') {
      c->p++;
      continue;
    }
    if (c->p < c->end && *c->p == close) {
      c->p++;
      return;
    }
    die_at(c, object ? "expected ',' or '}'" : "expected ',' or ']'");
  }
}

static void parse_value(cursor_t* c, json_value_t* v, int depth) {
  if (depth > 256) {
    die_at(c, "nesting too deep");
  }
  skip_space(c);
  if (c->p >= c->end) {
    die_at(c, "unexpected end of input");
  }
  v->line = c->line;
  char ch = *c->p;
  if (ch == '{' || ch == '[') {
    parse_container(c, v, depth);
  } else if (ch == '"') {
    v->kind = JSON_STRING;
    v->string = parse_string_raw(c);
  } else if (ch == '-' || ch == '+' || ch == '.' || is_digit(ch)) {
    parse_number(c, v);
  } else if (match_word(c, "true")) {
    v->kind = JSON_BOOL;
    v->boolean = true;
  } else if (match_word(c, "false")) {
    v->kind = JSON_BOOL;
    v->boolean = false;
  } else if (match_word(c, "null")) {
    v->kind = JSON_NULL;
  } else {
    die_at(c, "unexpected character");
  }
}

json_value_t* json_parse(const char* text, size_t len, const char* what) {
  cursor_t c = {text, text + len, 1, what ? what : "json"};
  json_value_t* v = calloc(1, sizeof(*v));
  if (!v) {
    die_at(&c, "out of host memory");
  }
  parse_value(&c, v, 0);
  return v;
}

json_value_t* json_parse_file(const char* path) {
  FILE* f = fopen(path, "rb");
  if (!f) {
    return NULL;
  }
  if (fseek(f, 0, SEEK_END) != 0) {
    fclose(f);
    return NULL;
  }
  long n = ftell(f);
  if (n < 0 || fseek(f, 0, SEEK_SET) != 0) {
    fclose(f);
    return NULL;
  }
  char* buf = malloc((size_t)n + 1);
  if (!buf) {
    fclose(f);
    return NULL;
  }
  size_t got = fread(buf, 1, (size_t)n, f);
  fclose(f);
  if (got != (size_t)n) {
    free(buf);
    return NULL;
  }
  buf[n] = '\0';
  json_value_t* v = json_parse(buf, (size_t)n, path);
  free(buf);
  return v;
}

static void free_children(json_value_t* v) {
  if (v->kind == JSON_STRING) {
    free(v->string);
  }
  if (v->kind == JSON_ARRAY || v->kind == JSON_OBJECT) {
    for (size_t i = 0; i < v->count; i++) {
      free_children(&v->item[i]);
      if (v->kind == JSON_OBJECT) {
        free(v->key[i]);
      }
    }
    free(v->item);
    free(v->key);
  }
}

void json_free(json_value_t* v) {
  if (v) {
    free_children(v);
    free(v);
  }
}

const json_value_t* json_get(const json_value_t* v, const char* key) {
  if (!v || v->kind != JSON_OBJECT) {
    return NULL;
  }
  for (size_t i = 0; i < v->count; i++) {
    if (strcmp(v->key[i], key) == 0) {
      return &v->item[i];
    }
  }
  return NULL;
}
