/* emmy_irdecode.c -- native decoder of the Kernel IR statement repr (module _irdecode).
 *
 * A KernelOp body is stored as Python repr text built from the IR constructors
 * (Tile(...), Load(...), BinaryExpr(...), ...). emmyptx/ir.py decodes it in pure
 * Python (a regex rewrite to JSON, or the ast module); for the large matmul and
 * attention bodies (150-200 KB of text) that is most of a compile. This module
 * reads the same grammar in one pass in C and builds the same node objects:
 *
 *   call    := NAME '(' [arg (',' arg)* [',']] ')'     NAME a registered constructor
 *   arg     := NAME '=' value | value
 *   value   := call | '(' values ')' | '[' values ']'  (both become tuples)
 *            | 'text' | number | None | True | False | inf | nan | -inf
 *
 * Identical call texts are decoded once and the node is shared (nodes are
 * immutable): before parsing a call, its closing parenthesis is found and the
 * exact text is looked up in a memo. Anything outside this subset (double
 * quotes, backslashes, non-ASCII text, unknown bare names) raises
 * _irdecode.Fallback, and a grammar error inside it raises the IRDecodeError
 * given to setup(); ir.py then decodes the statement with its Python decoders,
 * which are the reference for the result and for the error messages.
 *
 * Values nest at most MAX_DEPTH levels (real bodies nest a few tens): the parser
 * recurses once per level, and a deeper text raises Fallback before the C stack
 * could overflow, so a malformed IR file ends in a decode error, not a crash.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>

#include <stdlib.h>
#include <string.h>

#define MAX_DEPTH 1000

static PyObject *g_classes;   /* name -> class */
static PyObject *g_fields;    /* name -> tuple of field names */
static PyObject *g_defaults;  /* name -> {field: default} */
static PyObject *g_decode_error;
static PyObject *g_fallback;
static PyObject *g_empty;     /* () */

typedef struct {
  const char *s;
  Py_ssize_t n, i;
  int depth;      /* values being parsed around the current position */
  PyObject *memo; /* call text -> node */
} P;

static PyObject *fallback(const char *why) {
  PyErr_SetString(g_fallback, why);
  return NULL;
}

static void skip_ws(P *p) {
  while (p->i < p->n && (p->s[p->i] == ' ' || p->s[p->i] == '\n' || p->s[p->i] == '\t' ||
                         p->s[p->i] == '\r'))
    p->i++;
}

static int is_ident_start(char c) {
  return (c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || c == '_';
}

static int is_ident(char c) { return is_ident_start(c) || (c >= '0' && c <= '9'); }

/* index just past the ')' closing the '(' at position open, or -1 */
static Py_ssize_t match_paren(const P *p, Py_ssize_t open) {
  int depth = 0;
  for (Py_ssize_t j = open; j < p->n; ++j) {
    char c = p->s[j];
    if (c == '\'') {
      ++j;
      while (j < p->n && p->s[j] != '\'') ++j;
      if (j >= p->n) return -1;
    } else if (c == '(' || c == '[') {
      ++depth;
    } else if (c == ')' || c == ']') {
      if (--depth == 0) return j + 1;
    }
  }
  return -1;
}

static PyObject *parse_value(P *p);

/* '(' or '[' sequence -> tuple */
static PyObject *parse_seq(P *p, char close) {
  p->i++; /* opening bracket */
  PyObject *list = PyList_New(0);
  if (!list) return NULL;
  int trailing_comma = 0;
  for (;;) {
    skip_ws(p);
    if (p->i >= p->n) {
      Py_DECREF(list);
      return fallback("unterminated sequence");
    }
    if (p->s[p->i] == close) {
      p->i++;
      break;
    }
    trailing_comma = 0;
    PyObject *v = parse_value(p);
    if (!v) {
      Py_DECREF(list);
      return NULL;
    }
    int rc = PyList_Append(list, v);
    Py_DECREF(v);
    if (rc) {
      Py_DECREF(list);
      return NULL;
    }
    skip_ws(p);
    if (p->i < p->n && p->s[p->i] == ',') {
      p->i++;
      trailing_comma = 1;
    } else if (p->i >= p->n || p->s[p->i] != close) {
      Py_DECREF(list);
      return fallback("malformed sequence");
    }
  }
  /* '(v)' is v itself in Python but a one-element list on the JSON path: a repr never
     writes it, so the Python decoders decide */
  if (close == ')' && PyList_GET_SIZE(list) == 1 && !trailing_comma) {
    Py_DECREF(list);
    return fallback("parenthesized value");
  }
  PyObject *t = PyList_AsTuple(list);
  Py_DECREF(list);
  return t;
}

static PyObject *parse_string(P *p) {
  Py_ssize_t a = ++p->i;
  while (p->i < p->n && p->s[p->i] != '\'') {
    if (p->s[p->i] == '\\') return fallback("escaped string");
    p->i++;
  }
  if (p->i >= p->n) return fallback("unterminated string");
  PyObject *u = PyUnicode_FromStringAndSize(p->s + a, p->i - a);
  p->i++;
  return u;
}

static PyObject *parse_number(P *p) {
  Py_ssize_t a = p->i;
  int is_float = 0;
  /* the grammar a repr writes: digits, '-' digits, -inf, -nan; a '+' sign, a lone '-' and
     leading zeros (which Python refuses in integers) are left to the Python decoders */
  if (p->s[p->i] == '+') return fallback("plus sign");
  if (p->s[p->i] == '-') p->i++;
  if (p->i >= p->n || !(is_ident_start(p->s[p->i]) || (p->s[p->i] >= '0' && p->s[p->i] <= '9')))
    return fallback("sign without a number");
  if (p->s[p->i] == '0' && p->i + 1 < p->n && p->s[p->i + 1] >= '0' && p->s[p->i + 1] <= '9')
    return fallback("leading zero");
  if (is_ident_start(p->s[p->i])) { /* -inf, -nan */
    Py_ssize_t b = p->i;
    while (p->i < p->n && is_ident(p->s[p->i])) p->i++;
    Py_ssize_t len = p->i - b;
    if (len == 3 && !memcmp(p->s + b, "inf", 3)) return PyFloat_FromDouble(-Py_HUGE_VAL);
    if (len == 3 && !memcmp(p->s + b, "nan", 3)) return PyFloat_FromDouble(-Py_NAN);
    return fallback("signed name");
  }
  while (p->i < p->n) {
    char c = p->s[p->i];
    if (c >= '0' && c <= '9') {
      p->i++;
    } else if (c == '.' || c == 'e' || c == 'E') {
      is_float = 1;
      p->i++;
    } else if ((c == '-' || c == '+') && (p->s[p->i - 1] == 'e' || p->s[p->i - 1] == 'E')) {
      p->i++;
    } else {
      break;
    }
  }
  Py_ssize_t len = p->i - a;
  if (len <= 0 || len > 64) return fallback("number");
  char buf[72];
  memcpy(buf, p->s + a, (size_t)len);
  buf[len] = '\0';
  if (is_float) {
    char *end = NULL;
    double v = strtod(buf, &end);
    if (end != buf + len) return fallback("number");
    return PyFloat_FromDouble(v);
  }
  return PyLong_FromString(buf, NULL, 10);
}

static PyObject *decode_error(const char *fmt, PyObject *a, PyObject *b) {
  PyErr_Format(g_decode_error, fmt, a, b);
  return NULL;
}

/* NAME '(' ... ')' starting at p->i (on the name); name spans [a, b) */
static PyObject *parse_call(P *p, Py_ssize_t a, Py_ssize_t b) {
  Py_ssize_t end = match_paren(p, b);
  if (end < 0) return fallback("unbalanced call");
  PyObject *key = PyUnicode_FromStringAndSize(p->s + a, end - a);
  if (!key) return NULL;
  PyObject *hit = PyDict_GetItemWithError(p->memo, key);
  if (hit) {
    Py_DECREF(key);
    Py_INCREF(hit);
    p->i = end;
    return hit;
  }
  if (PyErr_Occurred()) {
    Py_DECREF(key);
    return NULL;
  }
  PyObject *name = PyUnicode_FromStringAndSize(p->s + a, b - a);
  PyObject *cls = name ? PyDict_GetItemWithError(g_classes, name) : NULL;
  PyObject *fields = cls ? PyDict_GetItemWithError(g_fields, name) : NULL;
  if (!cls || !fields) {
    if (!PyErr_Occurred()) PyErr_Format(g_decode_error, "unknown IR constructor: %U", name);
    Py_XDECREF(name);
    Py_DECREF(key);
    return NULL;
  }
  Py_ssize_t nf = PyTuple_GET_SIZE(fields);
  PyObject *vals[32] = {0};
  PyObject *result = NULL;
  Py_ssize_t npos = 0;
  int kw_seen = 0;
  if (nf > 32) {
    fallback("too many fields");
    goto done;
  }
  p->i = b + 1; /* past '(' */
  for (;;) {
    skip_ws(p);
    if (p->i >= p->n) {
      fallback("unterminated call");
      goto done;
    }
    if (p->s[p->i] == ')') {
      p->i++;
      break;
    }
    /* keyword argument? */
    Py_ssize_t k0 = p->i, k1 = p->i;
    while (k1 < p->n && is_ident(p->s[k1])) k1++;
    Py_ssize_t k2 = k1;
    while (k2 < p->n && p->s[k2] == ' ') k2++;
    if (k1 > k0 && is_ident_start(p->s[k0]) && k2 < p->n && p->s[k2] == '=' &&
        (k2 + 1 >= p->n || p->s[k2 + 1] != '=')) {
      PyObject *kname = PyUnicode_FromStringAndSize(p->s + k0, k1 - k0);
      if (!kname) goto done;
      Py_ssize_t idx = -1;
      for (Py_ssize_t f = 0; f < nf; ++f) {
        int eq = PyUnicode_Compare(PyTuple_GET_ITEM(fields, f), kname);
        if (eq == 0) {
          idx = f;
          break;
        }
      }
      if (idx < 0) {
        decode_error("%U has no field %R", name, kname);
        Py_DECREF(kname);
        goto done;
      }
      if (vals[idx]) {
        decode_error("%U got %R twice", name, kname);
        Py_DECREF(kname);
        goto done;
      }
      Py_DECREF(kname);
      p->i = k2 + 1;
      PyObject *v = parse_value(p);
      if (!v) goto done;
      vals[idx] = v;
      kw_seen = 1;
    } else {
      if (kw_seen) {
        fallback("positional after keyword");
        goto done;
      }
      if (npos >= nf) {
        PyErr_Format(g_decode_error, "%U takes at most %zd positional arguments", name, nf);
        goto done;
      }
      PyObject *v = parse_value(p);
      if (!v) goto done;
      vals[npos++] = v;
    }
    skip_ws(p);
    if (p->i < p->n && p->s[p->i] == ',') {
      p->i++;
    } else if (p->i >= p->n || p->s[p->i] != ')') {
      fallback("malformed call");
      goto done;
    }
  }
  PyObject *defaults = PyDict_GetItemWithError(g_defaults, name);
  if (!defaults && PyErr_Occurred()) goto done;
  for (Py_ssize_t f = 0; f < nf; ++f) {
    if (vals[f]) continue;
    PyObject *d = defaults ? PyDict_GetItemWithError(defaults, PyTuple_GET_ITEM(fields, f)) : NULL;
    if (!d) {
      if (!PyErr_Occurred())
        decode_error("%U is missing field %R", name, PyTuple_GET_ITEM(fields, f));
      goto done;
    }
    Py_INCREF(d);
    vals[f] = d;
  }
  {
    PyObject *obj = PyBaseObject_Type.tp_new((PyTypeObject *)cls, g_empty, NULL);
    if (!obj) goto done;
    for (Py_ssize_t f = 0; f < nf; ++f) {
      if (PyObject_GenericSetAttr(obj, PyTuple_GET_ITEM(fields, f), vals[f])) {
        Py_DECREF(obj);
        goto done;
      }
    }
    if (PyDict_SetItem(p->memo, key, obj)) {
      Py_DECREF(obj);
      goto done;
    }
    result = obj;
  }
  if (p->i != end) { /* the scan and the parse must agree on the call's extent */
    Py_DECREF(result);
    result = fallback("call extent");
  }
done:
  for (Py_ssize_t f = 0; f < nf && f < 32; ++f) Py_XDECREF(vals[f]);
  Py_DECREF(name);
  Py_DECREF(key);
  return result;
}

static PyObject *parse_value_at(P *p) {
  skip_ws(p);
  if (p->i >= p->n) return fallback("unexpected end");
  char c = p->s[p->i];
  if (c == '(') return parse_seq(p, ')');
  if (c == '[') return parse_seq(p, ']');
  if (c == '\'') return parse_string(p);
  if (c == '"') return fallback("double-quoted string");
  if ((c >= '0' && c <= '9') || c == '-' || c == '+') return parse_number(p);
  if (is_ident_start(c)) {
    Py_ssize_t a = p->i;
    while (p->i < p->n && is_ident(p->s[p->i])) p->i++;
    Py_ssize_t b = p->i;
    if (b < p->n && p->s[b] == '(') return parse_call(p, a, b);
    Py_ssize_t len = b - a;
    if (len == 4 && !memcmp(p->s + a, "None", 4)) Py_RETURN_NONE;
    if (len == 4 && !memcmp(p->s + a, "True", 4)) Py_RETURN_TRUE;
    if (len == 5 && !memcmp(p->s + a, "False", 5)) Py_RETURN_FALSE;
    if (len == 3 && !memcmp(p->s + a, "inf", 3)) return PyFloat_FromDouble(Py_HUGE_VAL);
    if (len == 3 && !memcmp(p->s + a, "nan", 3)) return PyFloat_FromDouble(Py_NAN);
    return fallback("bare name");
  }
  return fallback("unexpected character");
}

static PyObject *parse_value(P *p) {
  if (p->depth >= MAX_DEPTH) return fallback("nesting too deep");
  p->depth++;
  PyObject *v = parse_value_at(p);
  p->depth--;
  return v;
}

static PyObject *py_setup(PyObject *self, PyObject *args) {
  PyObject *classes, *fields, *defaults, *err;
  if (!PyArg_ParseTuple(args, "O!O!O!O", &PyDict_Type, &classes, &PyDict_Type, &fields,
                        &PyDict_Type, &defaults, &err))
    return NULL;
  Py_XSETREF(g_classes, Py_NewRef(classes));
  Py_XSETREF(g_fields, Py_NewRef(fields));
  Py_XSETREF(g_defaults, Py_NewRef(defaults));
  Py_XSETREF(g_decode_error, Py_NewRef(err));
  Py_RETURN_NONE;
}

static PyObject *py_decode(PyObject *self, PyObject *arg) {
  if (!g_classes) return fallback("not set up");
  if (!PyUnicode_Check(arg) || !PyUnicode_IS_ASCII(arg)) return fallback("not ASCII text");
  P p;
  p.s = (const char *)PyUnicode_1BYTE_DATA(arg);
  p.n = PyUnicode_GET_LENGTH(arg);
  p.i = 0;
  p.depth = 0;
  p.memo = PyDict_New();
  if (!p.memo) return NULL;
  PyObject *v = parse_value(&p);
  if (v) {
    skip_ws(&p);
    if (p.i != p.n) {
      Py_DECREF(v);
      v = fallback("trailing text");
    }
  }
  Py_DECREF(p.memo);
  return v;
}

static PyMethodDef methods[] = {
    {"setup", py_setup, METH_VARARGS,
     "setup(classes, fields, defaults, decode_error): the constructors to build."},
    {"decode", py_decode, METH_O, "decode(text) -> the IR value the repr text describes."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef moddef = {PyModuleDef_HEAD_INIT, "_irdecode",
                                    "Native decoder of the Kernel IR repr grammar.", -1, methods};

PyMODINIT_FUNC PyInit__irdecode(void) {
  PyObject *m = PyModule_Create(&moddef);
  if (!m) return NULL;
  g_fallback = PyErr_NewException("_irdecode.Fallback", NULL, NULL);
  g_empty = PyTuple_New(0);
  if (!g_fallback || !g_empty || PyModule_AddObjectRef(m, "Fallback", g_fallback) < 0) {
    Py_DECREF(m);
    return NULL;
  }
  return m;
}
